// Multi-tensor AdamW (decoupled weight decay, Loshchilov & Hutter 2019) over
// fp32 master weights, writing the bf16 shadow copy the GEMMs read in the same
// pass, so no separate cast kernel runs before the next forward.
//
// Work is described by a device table of tensors plus a list of
// (tensor, chunk) pairs built once on the host; one launch updates every
// parameter of a group.  Per element:
//   g = grad * inv_scale                       (loss-scale removal, optional)
//   p = p - lr * wd * p
//   m = b1 m + (1 - b1) g ;  v = b2 v + (1 - b2) g^2
//   p = p - (lr / (1 - b1^t)) * m / (sqrt(v) / sqrt(1 - b2^t) + eps)
// which is the update torch.optim.AdamW applies (the reference trainer's
// optimizer, examples/train_gpt.py:185).  When `skip` points at a nonzero
// float (an overflow found by the grad scaler) the kernel leaves everything
// untouched, without a host synchronisation.
//
// mode 1 only refreshes the bf16 shadows from the fp32 weights.
#include "md_sm100.cuh"

struct MdAdamEntry {
  float* p;
  const float* g;
  float* m;
  float* v;
  __nv_bfloat16* shadow;  // may be null
  long long n;
};

namespace md {
namespace optim {

constexpr int kChunk = 8192;  // ~13 waves at GPT-2 size: a short tail wave

__global__ void __launch_bounds__(256) adamw_kernel(const MdAdamEntry* __restrict__ table,
                                                    const int2* __restrict__ chunks, float lr, float b1, float b2,
                                                    float eps, float wd, float bc1, float bc2_sqrt,
                                                    const float* __restrict__ inv_scale,
                                                    const float* __restrict__ skip, int mode,
                                                    const float* __restrict__ hp) {
  pdl_trigger();  // the next kernel may launch now
  pdl_wait();     // global memory only after the previous kernel completed
  if (mode == 0 && skip != nullptr && *skip != 0.f) return;
  if (hp != nullptr) {
    // Graph-replayable form: learning rate and step count come from device
    // memory, and the bias corrections are computed here.
    lr = hp[0];
    const float t = hp[1];
    bc1 = 1.f - powf(b1, t);
    bc2_sqrt = sqrtf(1.f - powf(b2, t));
  }
  const int2 c = chunks[blockIdx.x];
  const MdAdamEntry e = table[c.x];
  const long long lo = static_cast<long long>(c.y) * kChunk;
  const long long hi = lo + kChunk < e.n ? lo + kChunk : e.n;
  const float gs = inv_scale != nullptr ? *inv_scale : 1.f;
  const float step = lr / bc1;
  const float decay = 1.f - lr * wd;
  const bool vec = ((reinterpret_cast<uintptr_t>(e.p) | reinterpret_cast<uintptr_t>(e.g) |
                     reinterpret_cast<uintptr_t>(e.m) | reinterpret_cast<uintptr_t>(e.v)) & 15u) == 0 &&
                   (e.shadow == nullptr || (reinterpret_cast<uintptr_t>(e.shadow) & 7u) == 0) && (lo % 4 == 0);
  if (vec) {
    const long long nv = (hi - lo) / 4;
    for (long long i = threadIdx.x; i < nv; i += blockDim.x) {
      const long long k = lo + 4 * i;
      float4 p = *reinterpret_cast<const float4*>(e.p + k);
      if (mode == 0) {
        const float4 g = *reinterpret_cast<const float4*>(e.g + k);
        float4 m = *reinterpret_cast<const float4*>(e.m + k);
        float4 v = *reinterpret_cast<const float4*>(e.v + k);
        float* pp = &p.x;
        float* mm = &m.x;
        float* vv = &v.x;
        const float* gg = &g.x;
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const float gq = gg[q] * gs;
          mm[q] = b1 * mm[q] + (1.f - b1) * gq;
          vv[q] = b2 * vv[q] + (1.f - b2) * gq * gq;
          pp[q] = pp[q] * decay - step * mm[q] / (sqrtf(vv[q]) / bc2_sqrt + eps);
        }
        *reinterpret_cast<float4*>(e.p + k) = p;
        *reinterpret_cast<float4*>(e.m + k) = m;
        *reinterpret_cast<float4*>(e.v + k) = v;
      }
      if (e.shadow != nullptr) {
        uint2 o;
        o.x = pack_bf16x2(p.x, p.y);
        o.y = pack_bf16x2(p.z, p.w);
        *reinterpret_cast<uint2*>(e.shadow + k) = o;
      }
    }
    for (long long k = lo + 4 * nv + threadIdx.x; k < hi; k += blockDim.x) {
      float pv = e.p[k];
      if (mode == 0) {
        const float gq = e.g[k] * gs;
        const float mv = b1 * e.m[k] + (1.f - b1) * gq;
        const float vv = b2 * e.v[k] + (1.f - b2) * gq * gq;
        pv = pv * decay - step * mv / (sqrtf(vv) / bc2_sqrt + eps);
        e.p[k] = pv;
        e.m[k] = mv;
        e.v[k] = vv;
      }
      if (e.shadow != nullptr) e.shadow[k] = __float2bfloat16_rn(pv);
    }
  } else {
    for (long long k = lo + threadIdx.x; k < hi; k += blockDim.x) {
      float pv = e.p[k];
      if (mode == 0) {
        const float gq = e.g[k] * gs;
        const float mv = b1 * e.m[k] + (1.f - b1) * gq;
        const float vv = b2 * e.v[k] + (1.f - b2) * gq * gq;
        pv = pv * decay - step * mv / (sqrtf(vv) / bc2_sqrt + eps);
        e.p[k] = pv;
        e.m[k] = mv;
        e.v[k] = vv;
      }
      if (e.shadow != nullptr) e.shadow[k] = __float2bfloat16_rn(pv);
    }
  }
}

// Loss-scaler overflow test over the same (tensor, chunk) table: *flag = 1
// when any gradient element is inf or NaN (read-only; the unscale itself is
// folded into adamw_kernel through inv_scale, and the update is skipped
// there through `skip` = this flag after the cross-rank MAX).
__global__ void __launch_bounds__(256) nonfinite_kernel(const MdAdamEntry* __restrict__ table,
                                                        const int2* __restrict__ chunks, float* __restrict__ flag) {
  pdl_trigger();
  pdl_wait();
  const int2 c = chunks[blockIdx.x];
  const MdAdamEntry e = table[c.x];
  const long long lo = static_cast<long long>(c.y) * kChunk;
  const long long hi = lo + kChunk < e.n ? lo + kChunk : e.n;
  bool bad = false;
  for (long long k = lo + threadIdx.x; k < hi; k += blockDim.x) bad |= !isfinite(e.g[k]);
  if (__syncthreads_or(bad) && threadIdx.x == 0) *flag = 1.f;
}

}  // namespace optim
}  // namespace md

extern "C" {

// *flag = 1 if any gradient of the table is non-finite (flag is not cleared here).
int md_nonfinite(const void* table, const void* chunks, int num_chunks, float* flag, cudaStream_t s) {
  if (num_chunks <= 0) return 0;
  if (flag == nullptr) return -1;
  md::launch_pdl(md::optim::nonfinite_kernel, dim3(num_chunks), dim3(256), 0, s,
                 reinterpret_cast<const MdAdamEntry*>(table), reinterpret_cast<const int2*>(chunks), flag);
  return static_cast<int>(cudaGetLastError());
}

int md_adamw_chunk() { return md::optim::kChunk; }
int md_adamw_entry_bytes() { return static_cast<int>(sizeof(MdAdamEntry)); }

// hp: null, or device [lr, step] (then lr / bc1 / bc2_sqrt are ignored).
int md_adamw(const void* table, const void* chunks, int num_chunks, float lr, float b1, float b2, float eps, float wd,
             float bc1, float bc2_sqrt, const float* inv_scale, const float* skip, int mode, cudaStream_t s,
             const float* hp) {
  if (num_chunks <= 0) return 0;
  md::launch_pdl(md::optim::adamw_kernel, dim3(num_chunks), dim3(256), 0, s, reinterpret_cast<const MdAdamEntry*>(table),
      reinterpret_cast<const int2*>(chunks), lr, b1, b2, eps, wd, bc1,
      bc2_sqrt, inv_scale, skip, mode, hp);
  return static_cast<int>(cudaGetLastError());
}

}  // extern "C"
