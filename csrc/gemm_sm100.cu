// Persistent warp-specialised bf16 GEMM for sm_100a: TMA -> shared memory ->
// tcgen05.mma (accumulator in TMEM) -> tcgen05.ld -> fused epilogue -> global.
//
//   D[M,N] = epilogue( sum_k A[m,k] * B[n,k] )
//
// A and B are bf16 and each may be K-major or MN-major in memory, which covers
// the three products of a linear layer without any transpose copies:
//   forward  y  = x  W^T : A = x  (K-major),  B = W (K-major)
//   dgrad    dx = dy W   : A = dy (K-major),  B = W (MN-major)
//   wgrad    dW = dy^T x : A = dy (MN-major), B = x (MN-major)
//
// CTA layout (192 threads, one CTA per SM, grid = min(#SMs, #work units)):
//   warp 0     : TMA producer (one thread) filling a 4-stage smem ring
//   warp 1     : TMEM allocator + MMA issuer (one thread)
//   warps 2..5 : epilogue; warp w reads TMEM lanes 32*(w%4) .. +31
// The 512 TMEM columns hold two 128x256 fp32 accumulators, so the epilogue of
// tile i overlaps the main loop of tile i+1.
//
// Epilogues (EpiMode):
//   kEpiBF16  : (+bias) (-> store pre-activation, GELU) (+residual) -> bf16
//   kEpiF32   : fp32 store, optionally D += acc (gradient accumulation); with
//               k_splits > 1 each split writes a partial slab of `workspace`
//               and md_splitk_reduce sums them in a fixed order
//   kEpiDGELU : acc * gelu'(pre-activation) -> bf16   (MLP backward)
//   kEpiCE    : bf16 logits plus per-(row, column-tile) max / sum-exp and the
//               target logit, for the fused cross-entropy
//
// This replaces the reference's F.linear calls (tensor_parallel.py:291,354
// via models/gpt.py) and, through kEpiCE, the logits half of
// _VocabParallelCrossEntropy (tensor_parallel.py:451-479).
#include <cudaTypedefs.h>

#include "md_sm100.cuh"

namespace md {
namespace gemm {

constexpr int BM = 128;
constexpr int BN = 256;
constexpr int BK = 64;
constexpr int kStages = 4;
constexpr int kThreads = 192;
constexpr int kABytes = BM * BK * 2;   // 16 KB
constexpr int kBBytes = BN * BK * 2;   // 32 KB
constexpr int kStageBytes = kABytes + kBBytes;
constexpr int kTmemCols = 512;
constexpr int kSmemBytes = 1024 /*align slack*/ + kStages * kStageBytes + 256 /*barriers*/;

enum EpiMode : int { kEpiBF16 = 0, kEpiF32 = 1, kEpiDGELU = 2, kEpiCE = 3 };

}  // namespace gemm
}  // namespace md

// Parameters shared with the Python binding (minidist/ops/_native.py mirrors
// this layout field for field).
struct MdGemmParams {
  const void* A;
  const void* B;
  void* D;
  long long lda, ldb, ldd;
  int M, N, K;
  int a_mn_major, b_mn_major;
  int epi;            // md::gemm::EpiMode
  float alpha;
  int beta;           // kEpiF32: 1 -> D += result
  int gelu;           // kEpiBF16: apply GELU (and store pre-activation in aux)
  const float* bias;  // [N] fp32 or null
  void* aux;          // bf16 [M, ldaux]: pre-activation out (kEpiBF16+gelu) / in (kEpiDGELU)
  long long ldaux;
  const void* resid;  // bf16 [M, ldres] residual added last (kEpiBF16)
  long long ldres;
  float* workspace;   // fp32 split-K partials, k_splits * M * ldws
  long long ldws;
  int k_splits;
  const long long* ce_target;  // int64 [M] (kEpiCE)
  float* ce_max;               // [tiles_n, M]
  float* ce_sum;               // [tiles_n, M]
  float* ce_tgt;               // [M]
  long long ce_col_offset;     // global column id of this shard's column 0
  int num_sms;                 // grid cap (0 -> all SMs)
  md::Status* status;
};

namespace md {
namespace gemm {

struct KParams {
  MdGemmParams p;
  int tiles_m, tiles_n, units, k_blocks, kb_per_split;
};

__device__ __forceinline__ void decode_unit(const KParams& kp, int u, int& tm, int& tn, int& split) {
  const int per_split = kp.tiles_m * kp.tiles_n;
  split = u / per_split;
  const int rem = u - split * per_split;
  tm = rem / kp.tiles_n;
  tn = rem - tm * kp.tiles_n;
}

template <bool A_MN, bool B_MN, int EPI>
__global__ void __launch_bounds__(kThreads, 1)
    gemm_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                const __grid_constant__ KParams kp) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sA = smem;
  uint8_t* sB = smem + kStages * kABytes;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + kStages * kStageBytes);
  uint64_t* full_bar = bars;                  // [kStages]
  uint64_t* empty_bar = bars + kStages;       // [kStages]
  uint64_t* tfull_bar = bars + 2 * kStages;   // [2]
  uint64_t* tempty_bar = bars + 2 * kStages + 2;  // [2]
  uint64_t* drain_bar = bars + 2 * kStages + 4;   // [1]
  uint32_t* tmem_base_slot = reinterpret_cast<uint32_t*>(bars + 2 * kStages + 5);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(bars + 2 * kStages + 6);

  const MdGemmParams& p = kp.p;
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&full_bar[s], 1);
      mbar_init(&empty_bar[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&tfull_bar[a], 1);
      mbar_init(&tempty_bar[a], 128);
    }
    mbar_init(drain_bar, 1);
    *abort_flag = 0;
    fence_mbar_init();
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
  }
  if (warp == 1) {
    tmem_alloc(tmem_base_slot, kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_base_slot;

  if (warp == 0 && lane == 0) {
    // ------------------------------------------------------------ producer
    int stage = 0;
    uint32_t phase = 0;
    int armed_phase[kStages];
    for (int s = 0; s < kStages; ++s) armed_phase[s] = -1;
    bool ok = true;
    for (int u = blockIdx.x; u < kp.units && ok; u += gridDim.x) {
      int tm, tn, split;
      decode_unit(kp, u, tm, tn, split);
      const int kb0 = split * kp.kb_per_split;
      const int kb1 = min(kp.k_blocks, kb0 + kp.kb_per_split);
      for (int kb = kb0; kb < kb1; ++kb) {
        if (!mbar_wait(&empty_bar[stage], phase ^ 1u, p.status, 10, abort_flag)) {
          ok = false;
          break;
        }
        mbar_arrive_expect_tx(&full_bar[stage], kStageBytes);
        armed_phase[stage] = static_cast<int>(phase);
        uint8_t* a_dst = sA + stage * kABytes;
        uint8_t* b_dst = sB + stage * kBBytes;
        if (!A_MN) {
          tma_load_2d(&tmA, &full_bar[stage], a_dst, kb * BK, tm * BM);
        } else {
#pragma unroll
          for (int c = 0; c < BM / 64; ++c)
            tma_load_2d(&tmA, &full_bar[stage], a_dst + c * (64 * BK * 2), tm * BM + c * 64, kb * BK);
        }
        if (!B_MN) {
          tma_load_2d(&tmB, &full_bar[stage], b_dst, kb * BK, tn * BN);
        } else {
#pragma unroll
          for (int c = 0; c < BN / 64; ++c)
            tma_load_2d(&tmB, &full_bar[stage], b_dst + c * (64 * BK * 2), tn * BN + c * 64, kb * BK);
        }
        if (++stage == kStages) {
          stage = 0;
          phase ^= 1u;
        }
      }
    }
    // Make sure no bulk copy into our shared memory is still in flight.
    for (int s = 0; s < kStages; ++s)
      if (armed_phase[s] >= 0) mbar_wait(&full_bar[s], static_cast<uint32_t>(armed_phase[s]), p.status, 11, nullptr);
  } else if (warp == 1 && lane == 0) {
    // ------------------------------------------------------------ MMA issuer
    constexpr uint32_t idesc = idesc_bf16_f32(BM, BN, A_MN, B_MN);
    int stage = 0;
    uint32_t phase = 0;
    int acc = 0;
    uint32_t acc_phase = 0;
    bool ok = true;
    for (int u = blockIdx.x; u < kp.units && ok; u += gridDim.x) {
      int tm, tn, split;
      decode_unit(kp, u, tm, tn, split);
      const int kb0 = split * kp.kb_per_split;
      const int kb1 = min(kp.k_blocks, kb0 + kp.kb_per_split);
      if (!mbar_wait(&tempty_bar[acc], acc_phase ^ 1u, p.status, 20, abort_flag)) break;
      tc_fence_after();
      const uint32_t d_tmem = tmem_base + static_cast<uint32_t>(acc * BN);
      for (int kb = kb0; kb < kb1; ++kb) {
        if (!mbar_wait(&full_bar[stage], phase, p.status, 21, abort_flag)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t a_addr = smem_u32(sA + stage * kABytes);
        const uint32_t b_addr = smem_u32(sB + stage * kBBytes);
#pragma unroll
        for (int k = 0; k < BK / 16; ++k) {
          uint64_t adesc, bdesc;
          if (!A_MN) adesc = sdesc_sw128(a_addr + k * 32, 16, 1024);
          else       adesc = sdesc_sw128(a_addr + k * 2048, 64 * BK * 2, 1024);
          if (!B_MN) bdesc = sdesc_sw128(b_addr + k * 32, 16, 1024);
          else       bdesc = sdesc_sw128(b_addr + k * 2048, 64 * BK * 2, 1024);
          umma_bf16_ss(d_tmem, adesc, bdesc, idesc, (kb > kb0 || k > 0) ? 1u : 0u);
        }
        umma_commit(&empty_bar[stage]);
        if (++stage == kStages) {
          stage = 0;
          phase ^= 1u;
        }
      }
      if (!ok) break;
      umma_commit(&tfull_bar[acc]);
      if (++acc == 2) {
        acc = 0;
        acc_phase ^= 1u;
      }
    }
    // Drain: wait for every MMA this thread issued before TMEM is released.
    umma_commit(drain_bar);
    mbar_wait(drain_bar, 0, p.status, 22, nullptr);
  } else if (warp >= 2) {
    // ------------------------------------------------------------ epilogue
    const int quarter = warp & 3;  // TMEM lane quarter this warp may access
    int acc = 0;
    uint32_t acc_phase = 0;
    for (int u = blockIdx.x; u < kp.units; u += gridDim.x) {
      int tm, tn, split;
      decode_unit(kp, u, tm, tn, split);
      if (!mbar_wait(&tfull_bar[acc], acc_phase, p.status, 30, abort_flag)) break;
      tc_fence_after();
      const int row = tm * BM + quarter * 32 + lane;
      const bool row_ok = row < p.M;
      const uint32_t t_row = tmem_base + (static_cast<uint32_t>(quarter * 32) << 16) + static_cast<uint32_t>(acc * BN);

      float ce_m = -INFINITY, ce_s = 0.f, ce_t = 0.f;
      bool ce_hit = false;
      long long tgt = -1;
      if (EPI == kEpiCE && row_ok) tgt = p.ce_target[row] - p.ce_col_offset;

#pragma unroll 1
      for (int c = 0; c < BN / 32; ++c) {
        uint32_t r[32];
        tmem_ld_32x32b_x32(t_row + c * 32, r);
        tmem_ld_wait();
        const int n0 = tn * BN + c * 32;
        if (!row_ok || n0 >= p.N) continue;
        const bool full = (n0 + 32 <= p.N);
        float v[32];
#pragma unroll
        for (int j = 0; j < 32; ++j) v[j] = __uint_as_float(r[j]) * p.alpha;

        if (EPI == kEpiBF16) {
          if (p.bias != nullptr) {
#pragma unroll
            for (int j = 0; j < 32; ++j) v[j] += (n0 + j < p.N) ? p.bias[n0 + j] : 0.f;
          }
          if (p.gelu) {
            __nv_bfloat16* aux = reinterpret_cast<__nv_bfloat16*>(p.aux) + row * p.ldaux + n0;
            if (full) {
#pragma unroll
              for (int q = 0; q < 4; ++q) {
                uint4 w;
                w.x = pack_bf16x2(v[q * 8 + 0], v[q * 8 + 1]);
                w.y = pack_bf16x2(v[q * 8 + 2], v[q * 8 + 3]);
                w.z = pack_bf16x2(v[q * 8 + 4], v[q * 8 + 5]);
                w.w = pack_bf16x2(v[q * 8 + 6], v[q * 8 + 7]);
                reinterpret_cast<uint4*>(aux)[q] = w;
              }
            } else {
              #pragma unroll
              for (int j = 0; j < 32; ++j)
                if (n0 + j < p.N) aux[j] = __float2bfloat16_rn(v[j]);
            }
#pragma unroll
            for (int j = 0; j < 32; ++j) {
              // GELU of the bf16-rounded pre-activation, exactly what the
              // backward pass will differentiate.
              float h = __bfloat162float(__float2bfloat16_rn(v[j]));
              v[j] = gelu_tanh(h);
            }
          }
          if (p.resid != nullptr) {
            const __nv_bfloat16* rs = reinterpret_cast<const __nv_bfloat16*>(p.resid) + row * p.ldres + n0;
            if (full) {
#pragma unroll
              for (int q = 0; q < 4; ++q) {
                uint4 w = reinterpret_cast<const uint4*>(rs)[q];
                float2 f0 = unpack_bf16x2(w.x), f1 = unpack_bf16x2(w.y), f2 = unpack_bf16x2(w.z),
                       f3 = unpack_bf16x2(w.w);
                v[q * 8 + 0] += f0.x; v[q * 8 + 1] += f0.y; v[q * 8 + 2] += f1.x; v[q * 8 + 3] += f1.y;
                v[q * 8 + 4] += f2.x; v[q * 8 + 5] += f2.y; v[q * 8 + 6] += f3.x; v[q * 8 + 7] += f3.y;
              }
            } else {
              #pragma unroll
              for (int j = 0; j < 32; ++j)
                if (n0 + j < p.N) v[j] += __bfloat162float(rs[j]);
            }
          }
        } else if (EPI == kEpiDGELU) {
          const __nv_bfloat16* hx = reinterpret_cast<const __nv_bfloat16*>(p.aux) + row * p.ldaux + n0;
          if (full) {
#pragma unroll
            for (int q = 0; q < 4; ++q) {
              uint4 w = reinterpret_cast<const uint4*>(hx)[q];
              float2 f0 = unpack_bf16x2(w.x), f1 = unpack_bf16x2(w.y), f2 = unpack_bf16x2(w.z),
                     f3 = unpack_bf16x2(w.w);
              v[q * 8 + 0] *= gelu_tanh_grad(f0.x); v[q * 8 + 1] *= gelu_tanh_grad(f0.y);
              v[q * 8 + 2] *= gelu_tanh_grad(f1.x); v[q * 8 + 3] *= gelu_tanh_grad(f1.y);
              v[q * 8 + 4] *= gelu_tanh_grad(f2.x); v[q * 8 + 5] *= gelu_tanh_grad(f2.y);
              v[q * 8 + 6] *= gelu_tanh_grad(f3.x); v[q * 8 + 7] *= gelu_tanh_grad(f3.y);
            }
          } else {
            #pragma unroll
            for (int j = 0; j < 32; ++j)
              if (n0 + j < p.N) v[j] *= gelu_tanh_grad(__bfloat162float(hx[j]));
          }
        }

        if (EPI == kEpiF32) {
          float* dst;
          bool add = false;
          if (p.k_splits > 1) {
            dst = p.workspace + (static_cast<long long>(split) * p.M + row) * p.ldws + n0;
          } else {
            dst = reinterpret_cast<float*>(p.D) + row * p.ldd + n0;
            add = p.beta != 0;
          }
          if (full) {
#pragma unroll
            for (int q = 0; q < 8; ++q) {
              float4 w = make_float4(v[q * 4 + 0], v[q * 4 + 1], v[q * 4 + 2], v[q * 4 + 3]);
              if (add) {
                float4 o = reinterpret_cast<const float4*>(dst)[q];
                w.x += o.x; w.y += o.y; w.z += o.z; w.w += o.w;
              }
              reinterpret_cast<float4*>(dst)[q] = w;
            }
          } else {
            #pragma unroll
            for (int j = 0; j < 32; ++j)
              if (n0 + j < p.N) dst[j] = add ? dst[j] + v[j] : v[j];
          }
        } else {
          __nv_bfloat16* dst = reinterpret_cast<__nv_bfloat16*>(p.D) + row * p.ldd + n0;
          if (EPI == kEpiCE) {
            // Round once; statistics use the same bf16 values the backward reads.
#pragma unroll
            for (int j = 0; j < 32; ++j) v[j] = __bfloat162float(__float2bfloat16_rn(v[j]));
            float cm = -INFINITY;
#pragma unroll
            for (int j = 0; j < 32; ++j)
              if (n0 + j < p.N) cm = fmaxf(cm, v[j]);
            if (cm > ce_m) {
              ce_s = (ce_m == -INFINITY) ? 0.f : ce_s * exp2f((ce_m - cm) * 1.4426950408889634f);
              ce_m = cm;
            }
            float s = 0.f;
#pragma unroll
            for (int j = 0; j < 32; ++j)
              if (n0 + j < p.N) s += exp2f((v[j] - ce_m) * 1.4426950408889634f);
            ce_s += s;
            if (tgt >= n0 && tgt < n0 + 32) {
#pragma unroll
              for (int j = 0; j < 32; ++j)
                if (n0 + j == tgt) ce_t = v[j];
              ce_hit = true;
            }
          }
          if (full) {
#pragma unroll
            for (int q = 0; q < 4; ++q) {
              uint4 w;
              w.x = pack_bf16x2(v[q * 8 + 0], v[q * 8 + 1]);
              w.y = pack_bf16x2(v[q * 8 + 2], v[q * 8 + 3]);
              w.z = pack_bf16x2(v[q * 8 + 4], v[q * 8 + 5]);
              w.w = pack_bf16x2(v[q * 8 + 6], v[q * 8 + 7]);
              reinterpret_cast<uint4*>(dst)[q] = w;
            }
          } else {
            #pragma unroll
            for (int j = 0; j < 32; ++j)
              if (n0 + j < p.N) dst[j] = __float2bfloat16_rn(v[j]);
          }
        }
      }
      if (EPI == kEpiCE && row_ok) {
        p.ce_max[static_cast<long long>(tn) * p.M + row] = ce_m;
        p.ce_sum[static_cast<long long>(tn) * p.M + row] = ce_s;
        if (ce_hit) p.ce_tgt[row] = ce_t;
      }
      tc_fence_before();
      mbar_arrive(&tempty_bar[acc]);
      if (++acc == 2) {
        acc = 0;
        acc_phase ^= 1u;
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) tmem_dealloc(tmem_base, kTmemCols);
}

// Fixed-order sum of split-K partials: D (+)= sum_s ws[s].  Deterministic, so
// replicated gradients stay bit-identical across ranks.
__global__ void splitk_reduce_kernel(const float* __restrict__ ws, float* __restrict__ D, long long ldd,
                                     long long ldws, int M, int N, int splits, int beta) {
  const long long total = static_cast<long long>(M) * N;
  for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<long long>(gridDim.x) * blockDim.x) {
    const long long m = i / N, n = i - m * N;
    float acc = beta ? D[m * ldd + n] : 0.f;
    for (int s = 0; s < splits; ++s) acc += ws[(static_cast<long long>(s) * M + m) * ldws + n];
    D[m * ldd + n] = acc;
  }
}

}  // namespace gemm
}  // namespace md

// ---------------------------------------------------------------------------
// Host side
// ---------------------------------------------------------------------------
namespace {

PFN_cuTensorMapEncodeTiled_v12000 g_encode = nullptr;

bool get_encoder() {
  if (g_encode != nullptr) return true;
  void* fn = nullptr;
  cudaDriverEntryPointQueryResult q;
  if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q) != cudaSuccess ||
      q != cudaDriverEntryPointSuccess || fn == nullptr)
    return false;
  g_encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
  return true;
}

// 2-D bf16 tensor map, 128-byte swizzle, box {64, box_outer}.
bool make_map(CUtensorMap* map, const void* ptr, uint64_t inner, uint64_t outer, uint64_t row_stride_elems,
              uint32_t box_outer) {
  cuuint64_t dims[2] = {inner, outer};
  cuuint64_t strides[1] = {row_stride_elems * 2};
  cuuint32_t box[2] = {64, box_outer};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = g_encode(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(ptr), dims, strides, box, estr,
                        CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                        CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

int g_num_sms = 0;

template <bool A_MN, bool B_MN, int EPI>
cudaError_t launch(const CUtensorMap& ta, const CUtensorMap& tb, const md::gemm::KParams& kp, int grid,
                   cudaStream_t stream) {
  auto kern = md::gemm::gemm_kernel<A_MN, B_MN, EPI>;
  static bool attr_set = false;  // per instantiation
  if (!attr_set) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, md::gemm::kSmemBytes);
    if (e != cudaSuccess) return e;
    attr_set = true;
  }
  kern<<<grid, md::gemm::kThreads, md::gemm::kSmemBytes, stream>>>(ta, tb, kp);
  return cudaGetLastError();
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

}  // namespace

// Return codes: 0 ok; negative = argument error (nothing launched); positive =
// CUDA error code from the launch.
extern "C" int md_gemm(const MdGemmParams* prm, cudaStream_t stream) {
  using namespace md::gemm;
  if (prm == nullptr) return -1;
  MdGemmParams p = *prm;
  if (p.M <= 0 || p.N <= 0 || p.K <= 0) return -2;
  if (!get_encoder()) return -3;
  if (!aligned16(p.A) || !aligned16(p.B) || (p.lda % 8) || (p.ldb % 8)) return -4;
  if (p.epi == kEpiF32) {
    if (!aligned16(p.D) || (p.ldd % 4)) return -5;
    if (p.k_splits > 1 && (p.workspace == nullptr || !aligned16(p.workspace) || (p.ldws % 4))) return -6;
  } else {
    if (!aligned16(p.D) || (p.ldd % 8)) return -5;
    if (p.k_splits != 1) return -6;
  }
  if (p.gelu && (p.aux == nullptr || !aligned16(p.aux) || (p.ldaux % 8))) return -7;
  if (p.epi == kEpiDGELU && (p.aux == nullptr || !aligned16(p.aux) || (p.ldaux % 8))) return -7;
  if (p.resid != nullptr && (!aligned16(p.resid) || (p.ldres % 8))) return -8;
  if (p.epi == kEpiCE && (p.ce_target == nullptr || p.ce_max == nullptr || p.ce_sum == nullptr || p.ce_tgt == nullptr))
    return -9;
  if (p.k_splits < 1) p.k_splits = 1;

  CUtensorMap ta, tb;
  bool ok;
  if (!p.a_mn_major) ok = make_map(&ta, p.A, p.K, p.M, p.lda, BM);
  else               ok = make_map(&ta, p.A, p.M, p.K, p.lda, 64);
  if (!ok) return -10;
  if (!p.b_mn_major) ok = make_map(&tb, p.B, p.K, p.N, p.ldb, BN);
  else               ok = make_map(&tb, p.B, p.N, p.K, p.ldb, 64);
  if (!ok) return -11;

  KParams kp;
  kp.p = p;
  kp.tiles_m = (p.M + BM - 1) / BM;
  kp.tiles_n = (p.N + BN - 1) / BN;
  kp.k_blocks = (p.K + BK - 1) / BK;
  if (p.k_splits > kp.k_blocks) p.k_splits = kp.k_blocks;
  kp.p.k_splits = p.k_splits;
  kp.kb_per_split = (kp.k_blocks + p.k_splits - 1) / p.k_splits;
  // Recompute the split count so that no split is empty.
  kp.p.k_splits = (kp.k_blocks + kp.kb_per_split - 1) / kp.kb_per_split;
  kp.units = kp.tiles_m * kp.tiles_n * kp.p.k_splits;

  if (g_num_sms == 0) {
    int dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&g_num_sms, cudaDevAttrMultiProcessorCount, dev);
  }
  int cap = p.num_sms > 0 ? p.num_sms : g_num_sms;
  int grid = kp.units < cap ? kp.units : cap;

  cudaError_t e;
  const bool amn = p.a_mn_major != 0, bmn = p.b_mn_major != 0;
  if (!amn && !bmn) {
    switch (p.epi) {
      case kEpiBF16: e = launch<false, false, kEpiBF16>(ta, tb, kp, grid, stream); break;
      case kEpiF32: e = launch<false, false, kEpiF32>(ta, tb, kp, grid, stream); break;
      case kEpiCE: e = launch<false, false, kEpiCE>(ta, tb, kp, grid, stream); break;
      default: return -12;
    }
  } else if (!amn && bmn) {
    switch (p.epi) {
      case kEpiBF16: e = launch<false, true, kEpiBF16>(ta, tb, kp, grid, stream); break;
      case kEpiF32: e = launch<false, true, kEpiF32>(ta, tb, kp, grid, stream); break;
      case kEpiDGELU: e = launch<false, true, kEpiDGELU>(ta, tb, kp, grid, stream); break;
      default: return -12;
    }
  } else if (amn && bmn) {
    switch (p.epi) {
      case kEpiF32: e = launch<true, true, kEpiF32>(ta, tb, kp, grid, stream); break;
      case kEpiBF16: e = launch<true, true, kEpiBF16>(ta, tb, kp, grid, stream); break;
      default: return -12;
    }
  } else {
    switch (p.epi) {
      case kEpiF32: e = launch<true, false, kEpiF32>(ta, tb, kp, grid, stream); break;
      case kEpiBF16: e = launch<true, false, kEpiBF16>(ta, tb, kp, grid, stream); break;
      default: return -12;
    }
  }
  if (e != cudaSuccess) return static_cast<int>(e);

  if (p.epi == kEpiF32 && kp.p.k_splits > 1) {
    const long long total = static_cast<long long>(p.M) * p.N;
    int blocks = static_cast<int>((total + 255) / 256);
    if (blocks > 4 * g_num_sms * 8) blocks = 4 * g_num_sms * 8;
    md::gemm::splitk_reduce_kernel<<<blocks, 256, 0, stream>>>(p.workspace, reinterpret_cast<float*>(p.D), p.ldd,
                                                               p.ldws, p.M, p.N, kp.p.k_splits, p.beta);
    e = cudaGetLastError();
    if (e != cudaSuccess) return static_cast<int>(e);
  }
  return 0;
}

// Number of CE partial column tiles the kEpiCE epilogue writes for N columns.
extern "C" int md_gemm_tile_n() { return md::gemm::BN; }
