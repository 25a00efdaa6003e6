// Token + position embedding, forward and backward, for bf16 activations.
//
// forward : out[m, :] = wte[ids[m] - vocab_start, :] (0 if the id is outside
//           this rank's vocabulary shard) + (add_pos ? wpe[m % S, :] : 0)
// backward: d_wte[id - vocab_start] += dx[m]   (fp32 vector atomics; rows are
//           rarely hit twice in one warp-step, so contention is low)
//           d_wpe[s] (+)= sum_b dx[b*S + s]    (fixed-order, deterministic)
//
// Reads the bf16 shadow of the tables; gradients land in fp32.
// Replaces VocabParallelEmbedding.forward (reference tensor_parallel.py:409-416)
// and Embedding.forward (models/gpt.py:183-185).
#include <atomic>

#include "md_noalloc.h"
#include "md_sm100.cuh"

namespace md {
namespace emb {

// One warp per token row; each lane moves 8 bf16 (16 B) per step.
__global__ void embed_fwd_kernel(const long long* __restrict__ ids, const __nv_bfloat16* __restrict__ wte,
                                 long long ldw, const __nv_bfloat16* __restrict__ wpe, long long ldp,
                                 __nv_bfloat16* __restrict__ out, long long ldo, int M, int S, int C,
                                 long long vocab_start, long long vocab_rows, int add_pos) {
  pdl_trigger();  // the next kernel may launch now
  pdl_wait();     // global memory only after the previous kernel completed
  const int warps = blockDim.x >> 5;
  const int lane = threadIdx.x & 31;
  const int nvec = C / 8;
  for (int m = blockIdx.x * warps + (threadIdx.x >> 5); m < M; m += gridDim.x * warps) {
    if (!MD_CHECK(ids[m] >= 0, MD_CHECK_STATUS, 300, ids[m])) continue;  // (rows of other shards are zero)
    const long long id = ids[m] - vocab_start;
    const bool own = id >= 0 && id < vocab_rows;
    const int s = m % S;
    for (int j = lane; j < nvec; j += 32) {
      float v[8];
      if (own) {
        const uint4 w = reinterpret_cast<const uint4*>(wte + id * ldw)[j];
        const uint32_t ws[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const float2 f = unpack_bf16x2(ws[q]);
          v[2 * q] = f.x;
          v[2 * q + 1] = f.y;
        }
      } else {
#pragma unroll
        for (int e = 0; e < 8; ++e) v[e] = 0.f;
      }
      if (add_pos) {
        const uint4 w = reinterpret_cast<const uint4*>(wpe + s * ldp)[j];
        const uint32_t ws[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const float2 f = unpack_bf16x2(ws[q]);
          v[2 * q] += f.x;
          v[2 * q + 1] += f.y;
        }
      }
      uint4 o;
      o.x = pack_bf16x2(v[0], v[1]);
      o.y = pack_bf16x2(v[2], v[3]);
      o.z = pack_bf16x2(v[4], v[5]);
      o.w = pack_bf16x2(v[6], v[7]);
      reinterpret_cast<uint4*>(out + m * ldo)[j] = o;
    }
  }
}

__global__ void embed_bwd_wte_kernel(const long long* __restrict__ ids, const __nv_bfloat16* __restrict__ dx,
                                     long long ldx, float* __restrict__ dwte, long long ldg, int M, int C,
                                     long long vocab_start, long long vocab_rows) {
  pdl_trigger();  // the next kernel may launch now
  pdl_wait();     // global memory only after the previous kernel completed
  const int warps = blockDim.x >> 5;
  const int lane = threadIdx.x & 31;
  const int nvec = C / 8;
  for (int m = blockIdx.x * warps + (threadIdx.x >> 5); m < M; m += gridDim.x * warps) {
    if (!MD_CHECK(ids[m] >= 0, MD_CHECK_STATUS, 301, ids[m])) continue;
    const long long id = ids[m] - vocab_start;
    if (id < 0 || id >= vocab_rows) continue;
    for (int j = lane; j < nvec; j += 32) {
      const uint4 w = reinterpret_cast<const uint4*>(dx + m * ldx)[j];
      const float2 a = unpack_bf16x2(w.x), b = unpack_bf16x2(w.y), c = unpack_bf16x2(w.z), d = unpack_bf16x2(w.w);
      float4* dst = reinterpret_cast<float4*>(dwte + id * ldg + j * 8);
      atomicAdd(dst, make_float4(a.x, a.y, b.x, b.y));
      atomicAdd(dst + 1, make_float4(c.x, c.y, d.x, d.y));
    }
  }
}

// d_wpe[s, c] (+)= sum_b dx[b*S + s, c]; one thread per (s, pair of columns).
__global__ void embed_bwd_wpe_kernel(const __nv_bfloat16* __restrict__ dx, long long ldx, float* __restrict__ dwpe,
                                     long long ldg, int B, int S, int C, int accumulate) {
  pdl_trigger();  // the next kernel may launch now
  pdl_wait();     // global memory only after the previous kernel completed
  const int pairs = C / 2;
  const long long total = static_cast<long long>(S) * pairs;
  for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<long long>(gridDim.x) * blockDim.x) {
    const int s = static_cast<int>(i / pairs);
    const int c2 = static_cast<int>(i - static_cast<long long>(s) * pairs);
    float ax = 0.f, ay = 0.f;
    for (int b = 0; b < B; ++b) {
      const uint32_t w = reinterpret_cast<const uint32_t*>(dx + (static_cast<long long>(b) * S + s) * ldx)[c2];
      const float2 f = unpack_bf16x2(w);
      ax += f.x;
      ay += f.y;
    }
    float2* dst = reinterpret_cast<float2*>(dwpe + s * ldg) + c2;
    if (accumulate) {
      float2 o = *dst;
      ax += o.x;
      ay += o.y;
    }
    *dst = make_float2(ax, ay);
  }
}

// Column sums of a bf16 matrix into fp32: out[n] (+)= sum_m x[m, n].
// Stage 1 writes one partial row per row-chunk, stage 2 adds them in order.
__global__ void colsum_partial_kernel(const __nv_bfloat16* __restrict__ x, long long ldx, int M, int N,
                                      int rows_per_chunk, float* __restrict__ partial) {
  pdl_trigger();  // the next kernel may launch now
  pdl_wait();     // global memory only after the previous kernel completed
  const int c2 = blockIdx.x * blockDim.x + threadIdx.x;  // column pair
  const int chunk = blockIdx.y;
  if (2 * c2 >= N) return;
  const int r0 = chunk * rows_per_chunk;
  const int r1 = min(M, r0 + rows_per_chunk);
  float ax = 0.f, ay = 0.f;
  const bool pair = 2 * c2 + 1 < N;
  for (int r = r0; r < r1; ++r) {
    if (pair) {
      const float2 f = unpack_bf16x2(reinterpret_cast<const uint32_t*>(x + r * ldx)[c2]);
      ax += f.x;
      ay += f.y;
    } else {
      ax += __bfloat162float(x[r * ldx + 2 * c2]);
    }
  }
  partial[static_cast<long long>(chunk) * N + 2 * c2] = ax;
  if (pair) partial[static_cast<long long>(chunk) * N + 2 * c2 + 1] = ay;
}

// Wide variant (N % 8 == 0, 16-byte aligned rows): a CTA covers 256 columns
// (32 groups of 8) x 8 row groups; the 8 row-group sums are added in a fixed
// order in shared memory, giving one partial row per (chunk, column block).
__global__ void __launch_bounds__(256) colsum_partial8_kernel(const __nv_bfloat16* __restrict__ x, long long ldx,
                                                              int M, int N, int rows_per_chunk,
                                                              float* __restrict__ partial) {
  pdl_trigger();  // the next kernel may launch now
  pdl_wait();     // global memory only after the previous kernel completed
  __shared__ float red[8][256 + 4];
  const int cgp = threadIdx.x & 31, rg = threadIdx.x >> 5;
  const int col = blockIdx.x * 256 + cgp * 8;
  const int chunk = blockIdx.y;
  const int r0 = chunk * rows_per_chunk;
  const int r1 = min(M, r0 + rows_per_chunk);
  float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
  if (col < N) {
    for (int r = r0 + rg; r < r1; r += 8) {
      const uint4 w = *reinterpret_cast<const uint4*>(x + r * ldx + col);
      const uint32_t ws[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const float2 f = unpack_bf16x2(ws[q]);
        acc[2 * q] += f.x;
        acc[2 * q + 1] += f.y;
      }
    }
  }
#pragma unroll
  for (int e = 0; e < 8; ++e) red[rg][cgp * 8 + e] = acc[e];
  __syncthreads();
  const int c = threadIdx.x;  // one output column per thread
  const int gc = blockIdx.x * 256 + c;
  if (gc < N) {
    float t = 0.f;
#pragma unroll
    for (int g = 0; g < 8; ++g) t += red[g][c];
    partial[static_cast<long long>(chunk) * N + gc] = t;
  }
}

// Second stage: out[n] (+)= sum over the partial rows.  A CTA covers 32
// columns with 32 warps; warp w takes rows w, w+32, ... (a few loads each, all
// in flight) and the 32 warp sums are added in a fixed order, so the result is
// deterministic and the pass costs about one memory latency.
__global__ void __launch_bounds__(1024) colsum_final_kernel(const float* __restrict__ partial, int chunks, int N,
                                                            float* __restrict__ out, int accumulate) {
  pdl_trigger();  // the next kernel may launch now
  pdl_wait();     // global memory only after the previous kernel completed
  __shared__ float red[32][33];
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  const int n = blockIdx.x * 32 + lane;
  float s = 0.f;
  if (n < N) {
    const float* col = partial + n;
#pragma unroll 4
    for (int c = w; c < chunks; c += 32) s += __ldg(col + static_cast<long long>(c) * N);
  }
  red[w][lane] = s;
  __syncthreads();
  if (w == 0 && n < N) {
    float t = 0.f;
#pragma unroll
    for (int g = 0; g < 32; ++g) t += red[g][lane];
    out[n] = accumulate ? out[n] + t : t;
  }
}

}  // namespace emb
}  // namespace md

namespace {
bool a16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }
}  // namespace

extern "C" {

int md_embed_fwd(const long long* ids, const void* wte, long long ldw, const void* wpe, long long ldp, void* out,
                 long long ldo, int M, int S, int C, long long vocab_start, long long vocab_rows, int add_pos,
                 cudaStream_t s) {
  if (M <= 0 || (C % 8) || (ldw % 8) || (ldo % 8) || !a16(wte) || !a16(out)) return -1;
  if (add_pos && ((ldp % 8) || !a16(wpe))) return -1;
  const int warps = 8;
  int grid = (M + warps - 1) / warps;
  if (grid > 148 * 16) grid = 148 * 16;
  md::launch_pdl(md::emb::embed_fwd_kernel, dim3(grid), dim3(warps * 32), 0, s,
      ids, reinterpret_cast<const __nv_bfloat16*>(wte), ldw, reinterpret_cast<const __nv_bfloat16*>(wpe), ldp,
      reinterpret_cast<__nv_bfloat16*>(out), ldo, M, S, C, vocab_start, vocab_rows, add_pos);
  return static_cast<int>(cudaGetLastError());
}

// d_wte must already hold the values to accumulate onto (zero it for a fresh gradient).
int md_embed_bwd_wte(const long long* ids, const void* dx, long long ldx, float* dwte, long long ldg, int M, int C,
                     long long vocab_start, long long vocab_rows, cudaStream_t s) {
  if (M <= 0 || (C % 8) || (ldx % 8) || (ldg % 4) || !a16(dx) || !a16(dwte)) return -1;
  const int warps = 8;
  int grid = (M + warps - 1) / warps;
  if (grid > 148 * 16) grid = 148 * 16;
  md::launch_pdl(md::emb::embed_bwd_wte_kernel, dim3(grid), dim3(warps * 32), 0, s, ids, reinterpret_cast<const __nv_bfloat16*>(dx), ldx,
      dwte, ldg, M, C, vocab_start, vocab_rows);
  return static_cast<int>(cudaGetLastError());
}

int md_embed_bwd_wpe(const void* dx, long long ldx, float* dwpe, long long ldg, int B, int S, int C, int accumulate,
                     cudaStream_t s) {
  if (B <= 0 || S <= 0 || (C % 2) || (ldx % 2) || (ldg % 2)) return -1;
  const long long total = static_cast<long long>(S) * (C / 2);
  int grid = static_cast<int>((total + 255) / 256);
  if (grid > 148 * 16) grid = 148 * 16;
  md::launch_pdl(md::emb::embed_bwd_wpe_kernel, dim3(grid), dim3(256), 0, s, reinterpret_cast<const __nv_bfloat16*>(dx), ldx, dwpe, ldg, B, S,
      C, accumulate);
  return static_cast<int>(cudaGetLastError());
}

// Number of row chunks (partial rows) md_colsum uses; the caller provides
// partial scratch of md_colsum_chunks(M, N) * N floats.
int md_colsum_chunks(int M, int N) {
  (void)N;
  int chunks = 148;
  const int max_chunks = (M + 63) / 64;
  if (chunks > max_chunks) chunks = max_chunks;
  return chunks < 1 ? 1 : chunks;
}

int md_colsum(const void* x, long long ldx, int M, int N, float* partial, float* out, int accumulate, cudaStream_t s) {
  if (M <= 0 || N <= 0 || (ldx % 2) || (reinterpret_cast<uintptr_t>(x) & 3u)) return -1;
  const int chunks = md_colsum_chunks(M, N);
  const int rows_per_chunk = (M + chunks - 1) / chunks;
  if ((N % 8) == 0 && (ldx % 8) == 0 && (reinterpret_cast<uintptr_t>(x) & 15u) == 0) {
    dim3 grid((N + 255) / 256, chunks);
    md::launch_pdl(md::emb::colsum_partial8_kernel, dim3(grid), dim3(256), 0, s, reinterpret_cast<const __nv_bfloat16*>(x), ldx, M, N,
        rows_per_chunk, partial);
  } else {
    dim3 grid((N / 2 + 1 + 255) / 256, chunks);
    md::launch_pdl(md::emb::colsum_partial_kernel, dim3(grid), dim3(256), 0, s, reinterpret_cast<const __nv_bfloat16*>(x), ldx, M, N,
        rows_per_chunk, partial);
  }
  md::launch_pdl(md::emb::colsum_final_kernel, dim3((N + 31) / 32), dim3(1024), 0, s, partial, chunks, N, out, accumulate);
  return static_cast<int>(cudaGetLastError());
}

// Second stage alone: out[n] (+)= sum_c partial[c * N + n] (first stages fused
// into producers, e.g. the GEMM's kEpiDGELU column sums).
int md_colsum_final(const float* partial, int chunks, int N, float* out, int accumulate, cudaStream_t s) {
  if (chunks <= 0 || N <= 0) return -1;
  md::launch_pdl(md::emb::colsum_final_kernel, dim3((N + 31) / 32), dim3(1024), 0, s, partial, chunks, N, out, accumulate);
  return static_cast<int>(cudaGetLastError());
}

}  // extern "C"

MD_DEFINE_CHECK_READER(md_check_status_embedding)

// ---------------------------------------------------------------------------
// Allocation-free variant of md_colsum (declared in md_noalloc.h).
//
// For callers that cannot allocate device memory themselves — for example a
// host program whose device memory is entirely owned by another allocator's
// pool, or code that must not call cudaMalloc because it may synchronise the
// device.  The partial-sum scratch of the two-stage column sum lives in the
// static array below, which every GPU that loads this library holds until the
// process exits.  Nothing in it needs clearing between calls: the first stage
// writes every scratch entry the second stage reads.
// ---------------------------------------------------------------------------
static __device__ __align__(256) float md_colsum_scratch[MD_NOALLOC_SCRATCH_FLOATS];

namespace {
constexpr int kMaxDevices = 64;
// Per-device device address of md_colsum_scratch, looked up on the first call
// on that device.  Atomic, so two host threads making their first call at the
// same time do not race (both store the same address).  A cudaDeviceReset
// ends the context the address belongs to; call md_colsum_noalloc_reset()
// after one so the next call looks the address up again.
std::atomic<void*> g_colsum_scratch[kMaxDevices];
}  // namespace

extern "C" long long md_colsum_scratch_floats(int M, int N) {
  if (M <= 0 || N <= 0) return 0;
  return static_cast<long long>(md_colsum_chunks(M, N)) * N;
}

extern "C" void md_colsum_noalloc_reset() {
  for (auto& a : g_colsum_scratch) a.store(nullptr, std::memory_order_release);
}

extern "C" int md_colsum_noalloc(const void* x, long long ldx, int M, int N, float* out, int accumulate,
                                 cudaStream_t s) {
  if (M <= 0 || N <= 0 || out == nullptr || x == nullptr) return -1;
  const long long need = static_cast<long long>(md_colsum_chunks(M, N)) * N;
  if (need > MD_NOALLOC_SCRATCH_FLOATS) return MD_NOALLOC_TOO_LARGE;
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return static_cast<int>(e);
  if (dev < 0 || dev >= kMaxDevices) return -2;
  void* scratch = g_colsum_scratch[dev].load(std::memory_order_acquire);
  if (scratch == nullptr) {
    // Device address of the static array for the current device; the host
    // symbol itself is only a stand-in and must never reach a kernel.
    e = cudaGetSymbolAddress(&scratch, md_colsum_scratch);
    if (e != cudaSuccess) return static_cast<int>(e);
    g_colsum_scratch[dev].store(scratch, std::memory_order_release);
  }
  return md_colsum(x, ldx, M, N, static_cast<float*>(scratch), out, accumulate, s);
}
