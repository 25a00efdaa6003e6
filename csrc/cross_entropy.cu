// Cross-entropy over (vocabulary-sharded) bf16 logits, in two small kernels
// around the LM-head GEMM, whose kEpiCE epilogue already produced, per row and
// per 256-column tile, the tile max and the sum of exp(z - tile max), plus the
// target logit when the target falls in this shard.
//
//   md_ce_stats    : combine the column tiles of each row into (max, sumexp)
//                    and, for an unsharded vocabulary, finish with
//                    lse = max + log(sumexp) and loss = lse - z_target.
//   md_ce_backward : dlogits = (exp(z - lse) - onehot(target)) * g / rows,
//                    recomputed from the stored bf16 logits, so the fp32
//                    softmax ([rows, V] floats) is never materialised.
//
// With tensor parallelism the per-row (max, sumexp, z_target) of each rank are
// combined across the group (MAX, rescaled SUM, SUM) before lse is formed —
// the decomposition of the reference's _VocabParallelCrossEntropy
// (tensor_parallel.py:451-492) with [rows]-sized instead of [rows, V]-sized
// intermediates.
#include "md_sm100.cuh"

namespace md {
namespace ce {

constexpr float kLog2e = 1.4426950408889634f;
constexpr float kLn2 = 0.6931471805599453f;

__global__ void stats_kernel(const float* __restrict__ tmax, const float* __restrict__ tsum, int tiles, int M,
                             float* __restrict__ row_max, float* __restrict__ row_sum,
                             const float* __restrict__ tgt_logit, float* __restrict__ lse_out,
                             float* __restrict__ loss_out) {
  pdl_trigger();  // the next kernel may launch now
  pdl_wait();     // global memory only after the previous kernel completed
  const int m = blockIdx.x * blockDim.x + threadIdx.x;
  if (m >= M) return;
  float mx = -INFINITY;
  for (int t = 0; t < tiles; ++t) mx = fmaxf(mx, tmax[static_cast<long long>(t) * M + m]);
  float s = 0.f;
  for (int t = 0; t < tiles; ++t) {
    const float tm = tmax[static_cast<long long>(t) * M + m];
    if (tm != -INFINITY) s += tsum[static_cast<long long>(t) * M + m] * exp2f((tm - mx) * kLog2e);
  }
  if (row_max) row_max[m] = mx;
  if (row_sum) row_sum[m] = s;
  if (lse_out) {
    const float lse = mx + log2f(s) * kLn2;
    lse_out[m] = lse;
    if (loss_out) loss_out[m] = lse - tgt_logit[m];
  }
}

// One CTA per row block; each thread handles 8 consecutive logits per vector,
// two vectors per step (both loads issued before either is used, so twice the
// bytes are in flight per thread: the kernel streams 2 x 1.65 GB at GPT-2 size).
__device__ __forceinline__ uint4 ce_grad8(uint4 w, int c0, float l, long long t, float g) {
  const uint32_t ws[4] = {w.x, w.y, w.z, w.w};
  uint32_t o[4];
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    const float2 f = unpack_bf16x2(ws[q]);
    const float p0 = exp2f((f.x - l) * kLog2e), p1 = exp2f((f.y - l) * kLog2e);
    o[q] = pack_bf16x2((p0 - ((c0 + 2 * q) == t ? 1.f : 0.f)) * g, (p1 - ((c0 + 2 * q + 1) == t ? 1.f : 0.f)) * g);
  }
  return make_uint4(o[0], o[1], o[2], o[3]);
}

__global__ void backward_kernel(const __nv_bfloat16* __restrict__ logits, long long ldl,
                                const float* __restrict__ lse, const long long* __restrict__ target,
                                long long col_offset, const float* __restrict__ grad_out, float scale,
                                __nv_bfloat16* __restrict__ dlogits, long long ldd, int M, int V) {
  pdl_trigger();  // the next kernel may launch now
  pdl_wait();     // global memory only after the previous kernel completed
  const float g = scale * (grad_out != nullptr ? grad_out[0] : 1.f);
  const int nfull = V / 8;  // whole 8-logit vectors; the ragged tail is done by thread 0
  const int nthr = static_cast<int>(blockDim.x);
  for (int m = blockIdx.x; m < M; m += gridDim.x) {
    const float l = lse[m];
    MD_CHECK(target[m] >= 0, MD_CHECK_STATUS, 310, target[m]);  // (a negative target matches no column)
    const long long t = target[m] - col_offset;
    const uint4* zr = reinterpret_cast<const uint4*>(logits + m * ldl);
    uint4* dr = reinterpret_cast<uint4*>(dlogits + m * ldd);
    for (int j = threadIdx.x; j < nfull; j += 2 * nthr) {
      const int j2 = j + nthr;
      const bool two = j2 < nfull;
      const uint4 w1 = zr[j];
      const uint4 w2 = two ? zr[j2] : make_uint4(0u, 0u, 0u, 0u);
      dr[j] = ce_grad8(w1, j * 8, l, t, g);
      if (two) dr[j2] = ce_grad8(w2, j2 * 8, l, t, g);
    }
    if (threadIdx.x == 0 && nfull * 8 < V) {
      const __nv_bfloat16* zs = logits + m * ldl;
      __nv_bfloat16* ds = dlogits + m * ldd;
      for (int c = nfull * 8; c < V; ++c) {
        const float p = exp2f((__bfloat162float(zs[c]) - l) * kLog2e);
        ds[c] = __float2bfloat16_rn((p - (c == t ? 1.f : 0.f)) * g);
      }
    }
  }
}

}  // namespace ce
}  // namespace md

extern "C" {

int md_ce_stats(const float* tmax, const float* tsum, int tiles, int M, float* row_max, float* row_sum,
                const float* tgt_logit, float* lse_out, float* loss_out, cudaStream_t s) {
  if (M <= 0 || tiles <= 0) return -1;
  md::launch_pdl(md::ce::stats_kernel, dim3((M + 255) / 256), dim3(256), 0, s, tmax, tsum, tiles, M, row_max, row_sum, tgt_logit, lse_out,
      loss_out);
  return static_cast<int>(cudaGetLastError());
}

int md_ce_backward(const void* logits, long long ldl, const float* lse, const long long* target, long long col_offset,
                   const float* grad_out, float scale, void* dlogits, long long ldd, int M, int V, cudaStream_t s) {
  if (M <= 0 || V <= 0 || (ldl % 8) || (ldd % 8) || (reinterpret_cast<uintptr_t>(logits) & 15u) ||
      (reinterpret_cast<uintptr_t>(dlogits) & 15u))
    return -1;
  int grid = M < 148 * 16 ? M : 148 * 16;
  md::launch_pdl(md::ce::backward_kernel, dim3(grid), dim3(256), 0, s, reinterpret_cast<const __nv_bfloat16*>(logits), ldl, lse, target,
      col_offset, grad_out, scale, reinterpret_cast<__nv_bfloat16*>(dlogits),
      ldd, M, V);
  return static_cast<int>(cudaGetLastError());
}

}  // extern "C"

MD_DEFINE_CHECK_READER(md_check_status_cross_entropy)
