// Causal flash attention (forward and backward) for bf16, head_dim in {64, 80, 128}.
//
// Q, K and V are read in place from the QKV projection output, whose columns
// are interleaved per head as [n_head, 3, head_dim] (reference
// models/gpt.py:92-99, 123-125), so no split/transpose copies run.  The output
// [tokens, n_head*head_dim] is the row-parallel projection's input as is, and
// the backward writes dQ/dK/dV into one buffer with the same interleaved
// layout, ready for the QKV weight-gradient and data-gradient GEMMs.
//
// Forward: one CTA per (128 queries, batch*head); 8 warps, 16 query rows each;
// K/V tiles of 64 keys double-buffered with cp.async; scores and the online
// softmax stay in registers; log-sum-exp per query row is saved for backward.
//
// Backward: one CTA per (64 keys, batch*head); 4 warps own 16 keys each and
// hold dK/dV in registers while sweeping the query blocks from the diagonal
// on.  Scores are recomputed transposed (S^T = K Q^T) so P^T and dS^T come out
// in the register layout the dV/dK products consume directly; dS^T is staged
// in shared memory for the dQ product, whose partial sums are added to an fp32
// accumulator with red.global.add (one 64 x head_dim tile per key block).
//
// This version uses the warp-level mma.sync tensor-core path.  Replaces
// F.scaled_dot_product_attention(is_causal=True) (reference models/gpt.py:126).
#include "md_sm100.cuh"

namespace md {
namespace attn {

__device__ __forceinline__ void cp_async16(void* smem, const void* gmem, bool valid) {
  const int n = valid ? 16 : 0;  // 0 bytes read -> zero fill
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(smem_u32(smem)), "l"(gmem), "r"(n) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

__device__ __forceinline__ void ldsm_x4(uint32_t (&r)[4], const void* p) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(smem_u32(p)));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t (&r)[4], const void* p) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(smem_u32(p)));
}
__device__ __forceinline__ void ldsm_x2_t(uint32_t (&r)[2], const void* p) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x2.trans.shared.b16 {%0, %1}, [%2];"
               : "=r"(r[0]), "=r"(r[1])
               : "r"(smem_u32(p)));
}
__device__ __forceinline__ void ldsm_x2(uint32_t (&r)[2], const void* p) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x2.shared.b16 {%0, %1}, [%2];"
               : "=r"(r[0]), "=r"(r[1])
               : "r"(smem_u32(p)));
}

// D += A * B for m16n8k16 bf16 with fp32 accumulators.
__device__ __forceinline__ void mma16816(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
      "{%0, %1, %2, %3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

__device__ __forceinline__ float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

constexpr float kLog2e = 1.4426950408889634f;
constexpr float kLn2 = 0.6931471805599453f;

// Copy a [rows x D] bf16 tile (global row stride ld) into padded shared rows
// (stride DP), zero-filling rows at or beyond `valid_rows`.
template <int D, int DP, int ROWS, int NTHREADS>
__device__ __forceinline__ void load_tile(__nv_bfloat16* s, const __nv_bfloat16* g, long long ld, int valid_rows) {
  constexpr int CPR = D / 8;  // 16-byte chunks per row
  for (int c = threadIdx.x; c < ROWS * CPR; c += NTHREADS) {
    const int r = c / CPR, k = c - r * CPR;
    const bool ok = r < valid_rows;
    cp_async16(s + r * DP + k * 8, g + (ok ? r : 0) * ld + k * 8, ok);
  }
}

// ============================================================================
// Forward
// ============================================================================
template <int D>
__global__ void __launch_bounds__(256) fwd_kernel(const __nv_bfloat16* __restrict__ qkv, long long ldq,
                                                  __nv_bfloat16* __restrict__ out, long long ldo,
                                                  float* __restrict__ lse_out, int H, int S, float scale_log2) {
  pdl_trigger();  // the next kernel may launch now
  pdl_wait();     // global memory only after the previous kernel completed
  constexpr int BM = 128, BN = 64, DP = D + 8, NT = D / 8, KS = D / 16;
  extern __shared__ __align__(16) __nv_bfloat16 fsm[];
  __nv_bfloat16* sQ = fsm;
  __nv_bfloat16* sK = sQ + BM * DP;
  __nv_bfloat16* sV = sK + 2 * BN * DP;

  const int mb = gridDim.x - 1 - blockIdx.x;  // heaviest (last) query blocks first
  const int bh = blockIdx.y, b = bh / H, h = bh - b * H;
  const int q0 = mb * BM;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, t = lane & 3;
  const __nv_bfloat16* base = qkv + static_cast<long long>(b) * S * ldq + h * 3 * D;

  load_tile<D, DP, BM, 256>(sQ, base + static_cast<long long>(q0) * ldq, ldq, S - q0);
  const int kv_end = min(S, q0 + BM);  // causal: keys < q0 + BM
  const int nblocks = (kv_end + BN - 1) / BN;
  load_tile<D, DP, BN, 256>(sK, base + D, ldq, S);
  load_tile<D, DP, BN, 256>(sV, base + 2 * D, ldq, S);
  cp_async_commit();

  float o[NT][4];
#pragma unroll
  for (int j = 0; j < NT; ++j) o[j][0] = o[j][1] = o[j][2] = o[j][3] = 0.f;
  float m0 = -INFINITY, m1 = -INFINITY, l0 = 0.f, l1 = 0.f;
  uint32_t qf[KS][4];
  const int qrow0 = q0 + warp * 16 + g;  // this thread's rows: qrow0 and qrow0 + 8

  for (int nb = 0; nb < nblocks; ++nb) {
    const int buf = nb & 1;
    if (nb + 1 < nblocks) {
      const int k1 = (nb + 1) * BN;
      load_tile<D, DP, BN, 256>(sK + (buf ^ 1) * BN * DP, base + static_cast<long long>(k1) * ldq + D, ldq, S - k1);
      load_tile<D, DP, BN, 256>(sV + (buf ^ 1) * BN * DP, base + static_cast<long long>(k1) * ldq + 2 * D, ldq,
                                S - k1);
      cp_async_commit();
      cp_async_wait<1>();
    } else {
      cp_async_wait<0>();
    }
    __syncthreads();
    if (nb == 0) {
#pragma unroll
      for (int ks = 0; ks < KS; ++ks)
        ldsm_x4(qf[ks], sQ + (warp * 16 + (lane & 15)) * DP + ks * 16 + (lane >> 4) * 8);
    }
    const __nv_bfloat16* k_s = sK + buf * BN * DP;
    const __nv_bfloat16* v_s = sV + buf * BN * DP;
    const int n0 = nb * BN;

    // S = Q K^T for this warp's 16 rows x 64 keys.
    float s[8][4];
#pragma unroll
    for (int j = 0; j < 8; ++j) s[j][0] = s[j][1] = s[j][2] = s[j][3] = 0.f;
    if (n0 <= q0 + warp * 16 + 15) {  // skip fully masked key blocks for this warp
#pragma unroll
      for (int ks = 0; ks < KS; ++ks) {
#pragma unroll
        for (int jp = 0; jp < 4; ++jp) {  // pairs of 8-key tiles
          uint32_t kb[4];
          ldsm_x4(kb, k_s + (jp * 16 + (lane & 7) + ((lane >> 4) << 3)) * DP + ks * 16 + ((lane >> 3) & 1) * 8);
          mma16816(s[2 * jp], qf[ks], kb[0], kb[1]);
          mma16816(s[2 * jp + 1], qf[ks], kb[2], kb[3]);
        }
      }
    }
    // Scale, mask (causal and sequence end), online softmax.
    const bool need_mask = (n0 + BN - 1 > q0 + warp * 16) || (n0 + BN > S);
    float mx0 = m0, mx1 = m1;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        float v = s[j][e] * scale_log2;
        if (need_mask) {
          const int key = n0 + 8 * j + 2 * t + (e & 1);
          const int q = qrow0 + ((e >> 1) << 3);
          if (key > q || key >= S) v = -INFINITY;
        }
        s[j][e] = v;
      }
      mx0 = fmaxf(mx0, fmaxf(s[j][0], s[j][1]));
      mx1 = fmaxf(mx1, fmaxf(s[j][2], s[j][3]));
    }
    mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 1));
    mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 2));
    mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 1));
    mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 2));
    const float c0 = (mx0 == -INFINITY) ? 1.f : ex2(m0 - mx0);
    const float c1 = (mx1 == -INFINITY) ? 1.f : ex2(m1 - mx1);
    const float base0 = (mx0 == -INFINITY) ? 0.f : mx0;
    const float base1 = (mx1 == -INFINITY) ? 0.f : mx1;
    float rs0 = 0.f, rs1 = 0.f;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      s[j][0] = ex2(s[j][0] - base0);
      s[j][1] = ex2(s[j][1] - base0);
      s[j][2] = ex2(s[j][2] - base1);
      s[j][3] = ex2(s[j][3] - base1);
      rs0 += s[j][0] + s[j][1];
      rs1 += s[j][2] + s[j][3];
    }
    l0 = l0 * c0 + rs0;
    l1 = l1 * c1 + rs1;
    m0 = mx0;
    m1 = mx1;
#pragma unroll
    for (int j = 0; j < NT; ++j) {
      o[j][0] *= c0;
      o[j][1] *= c0;
      o[j][2] *= c1;
      o[j][3] *= c1;
    }
    // O += P V  (P re-packed from the accumulator layout into A fragments).
#pragma unroll
    for (int kk = 0; kk < 4; ++kk) {
      uint32_t pa[4];
      pa[0] = pack_bf16x2(s[2 * kk][0], s[2 * kk][1]);
      pa[1] = pack_bf16x2(s[2 * kk][2], s[2 * kk][3]);
      pa[2] = pack_bf16x2(s[2 * kk + 1][0], s[2 * kk + 1][1]);
      pa[3] = pack_bf16x2(s[2 * kk + 1][2], s[2 * kk + 1][3]);
#pragma unroll
      for (int jp = 0; jp < NT / 2; ++jp) {
        uint32_t vb[4];
        ldsm_x4_t(vb, v_s + (kk * 16 + (lane & 7) + (((lane >> 3) & 1) << 3)) * DP + jp * 16 + (lane >> 4) * 8);
        mma16816(o[2 * jp], pa, vb[0], vb[1]);
        mma16816(o[2 * jp + 1], pa, vb[2], vb[3]);
      }
      if constexpr (NT % 2) {
        uint32_t vb[2];
        ldsm_x2_t(vb, v_s + (kk * 16 + (lane & 7) + (((lane >> 3) & 1) << 3)) * DP + (NT - 1) * 8);
        mma16816(o[NT - 1], pa, vb[0], vb[1]);
      }
    }
    __syncthreads();  // this buffer is refilled two iterations later
  }

  // Normalise, store O and the log-sum-exp (natural log) per row.
  l0 += __shfl_xor_sync(0xffffffffu, l0, 1);
  l0 += __shfl_xor_sync(0xffffffffu, l0, 2);
  l1 += __shfl_xor_sync(0xffffffffu, l1, 1);
  l1 += __shfl_xor_sync(0xffffffffu, l1, 2);
  const float inv0 = l0 > 0.f ? 1.f / l0 : 0.f;
  const float inv1 = l1 > 0.f ? 1.f / l1 : 0.f;
  const int r0 = qrow0, r1 = qrow0 + 8;
  __nv_bfloat16* ob = out + static_cast<long long>(b) * S * ldo + h * D;
#pragma unroll
  for (int j = 0; j < NT; ++j) {
    const int col = 8 * j + 2 * t;
    if (r0 < S)
      *reinterpret_cast<uint32_t*>(ob + static_cast<long long>(r0) * ldo + col) = pack_bf16x2(o[j][0] * inv0, o[j][1] * inv0);
    if (r1 < S)
      *reinterpret_cast<uint32_t*>(ob + static_cast<long long>(r1) * ldo + col) = pack_bf16x2(o[j][2] * inv1, o[j][3] * inv1);
  }
  if (t == 0) {
    float* lrow = lse_out + static_cast<long long>(bh) * S;
    if (r0 < S) lrow[r0] = (m0 + log2f(l0)) * kLn2;
    if (r1 < S) lrow[r1] = (m1 + log2f(l1)) * kLn2;
  }
}

// ============================================================================
// Backward preprocessing: delta[bh, q] = sum_d dO[q, d] * O[q, d]
// ============================================================================
template <int D>
__global__ void delta_kernel(const __nv_bfloat16* __restrict__ o, long long ldo, const __nv_bfloat16* __restrict__ dout,
                             long long lddo, float* __restrict__ delta, int B, int H, int S) {
  pdl_trigger();  // the next kernel may launch now
  pdl_wait();     // global memory only after the previous kernel completed
  if constexpr (D == 64 || D == 128) {
    // D/8 lanes per (row, head): each lane one 16-byte vector of O and dO
    // (consecutive lanes, consecutive bytes), then a shuffle reduction.
    constexpr int L = D / 8;
    constexpr int kItemsPerWarp = 32 / L;
    const long long total = static_cast<long long>(B) * H * S;
    const int lane = threadIdx.x & 31, sub = lane % L;
    const long long warp_id = (blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x) / 32;
    const long long warps = static_cast<long long>(gridDim.x) * blockDim.x / 32;
    // Warp-uniform loop (the shuffle needs every lane), predicated per item.
    for (long long base = warp_id * kItemsPerWarp; base < total; base += warps * kItemsPerWarp) {
      const long long i = base + lane / L;
      const bool valid = i < total;
      float acc = 0.f;
      long long bh = 0;
      int q = 0;
      if (valid) {
        q = static_cast<int>(i % S);
        bh = i / S;
        const int h = static_cast<int>(bh % H);
        const long long row = (bh / H) * S + q;
        const uint4 a = reinterpret_cast<const uint4*>(o + row * ldo + h * D)[sub];
        const uint4 c = reinterpret_cast<const uint4*>(dout + row * lddo + h * D)[sub];
        const uint32_t as[4] = {a.x, a.y, a.z, a.w}, cs[4] = {c.x, c.y, c.z, c.w};
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const float2 fa = unpack_bf16x2(as[e]), fc = unpack_bf16x2(cs[e]);
          acc += fa.x * fc.x + fa.y * fc.y;
        }
      }
#pragma unroll
      for (int off = L / 2; off > 0; off >>= 1) acc += __shfl_xor_sync(0xFFFFFFFFu, acc, off);
      if (valid && sub == 0) delta[bh * S + q] = acc;
    }
    return;
  }
  const long long total = static_cast<long long>(B) * H * S;
  for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<long long>(gridDim.x) * blockDim.x) {
    const int q = static_cast<int>(i % S);
    const long long bh = i / S;
    const int h = static_cast<int>(bh % H);
    const long long b = bh / H;
    const long long row = b * S + q;
    const uint4* po = reinterpret_cast<const uint4*>(o + row * ldo + h * D);
    const uint4* pd = reinterpret_cast<const uint4*>(dout + row * lddo + h * D);
    float acc = 0.f;
#pragma unroll
    for (int k = 0; k < D / 8; ++k) {
      const uint4 a = po[k], c = pd[k];
      const uint32_t as[4] = {a.x, a.y, a.z, a.w}, cs[4] = {c.x, c.y, c.z, c.w};
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float2 fa = unpack_bf16x2(as[e]), fc = unpack_bf16x2(cs[e]);
        acc += fa.x * fc.x + fa.y * fc.y;
      }
    }
    delta[bh * S + q] = acc;
  }
}

// dQ (bf16, in the interleaved QKV-gradient buffer) = scale * fp32 accumulator.
template <int D>
__global__ void dq_convert_kernel(const float* __restrict__ dqacc, long long lda, __nv_bfloat16* __restrict__ dqkv,
                                  long long lddq, int M, int H, float scale) {
  pdl_trigger();  // the next kernel may launch now
  pdl_wait();     // global memory only after the previous kernel completed
  if constexpr (D % 8 == 0) {
    // Eight elements per thread: two 16-byte loads, one 16-byte store.
    const long long total = static_cast<long long>(M) * H * (D / 8);
    for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < total;
         i += static_cast<long long>(gridDim.x) * blockDim.x) {
      const int c8 = static_cast<int>(i % (D / 8));
      const long long rh = i / (D / 8);
      const int h = static_cast<int>(rh % H);
      const long long row = rh / H;
      const float4* src = reinterpret_cast<const float4*>(dqacc + row * lda + h * D + 8 * c8);
      const float4 v0 = src[0], v1 = src[1];
      uint4 w;
      w.x = pack_bf16x2(v0.x * scale, v0.y * scale);
      w.y = pack_bf16x2(v0.z * scale, v0.w * scale);
      w.z = pack_bf16x2(v1.x * scale, v1.y * scale);
      w.w = pack_bf16x2(v1.z * scale, v1.w * scale);
      *reinterpret_cast<uint4*>(dqkv + row * lddq + h * 3 * D + 8 * c8) = w;
    }
    return;
  }
  const long long total = static_cast<long long>(M) * H * (D / 2);
  for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<long long>(gridDim.x) * blockDim.x) {
    const int c2 = static_cast<int>(i % (D / 2));
    const long long rh = i / (D / 2);
    const int h = static_cast<int>(rh % H);
    const long long row = rh / H;
    const float2 v = *reinterpret_cast<const float2*>(dqacc + row * lda + h * D + 2 * c2);
    *reinterpret_cast<uint32_t*>(dqkv + row * lddq + h * 3 * D + 2 * c2) = pack_bf16x2(v.x * scale, v.y * scale);
  }
}

__device__ __forceinline__ void red_add_f32x2(float* addr, float a, float b) {
  asm volatile("red.global.add.v2.f32 [%0], {%1, %2};" ::"l"(addr), "f"(a), "f"(b) : "memory");
}

// ============================================================================
// Backward main kernel
// ============================================================================
template <int D>
__global__ void __launch_bounds__(128) bwd_kernel(const __nv_bfloat16* __restrict__ qkv, long long ldq,
                                                  const __nv_bfloat16* __restrict__ dout, long long lddo,
                                                  const float* __restrict__ lse, const float* __restrict__ delta,
                                                  float* __restrict__ dqacc, long long ldacc,
                                                  __nv_bfloat16* __restrict__ dqkv, long long lddq, int H, int S,
                                                  float scale, float scale_log2) {
  pdl_trigger();  // the next kernel may launch now
  pdl_wait();     // global memory only after the previous kernel completed
  constexpr int BN = 64, BM = 64, DP = D + 8, NT = D / 8, KS = D / 16, SP = BM + 8;
  extern __shared__ __align__(16) __nv_bfloat16 bsm[];
  __nv_bfloat16* sK = bsm;                 // [BN][DP]
  __nv_bfloat16* sV = sK + BN * DP;        // [BN][DP]
  __nv_bfloat16* sQ = sV + BN * DP;        // [2][BM][DP]
  __nv_bfloat16* sdO = sQ + 2 * BM * DP;   // [2][BM][DP]
  __nv_bfloat16* sdS = sdO + 2 * BM * DP;  // [BN][SP]  (dS^T: keys x queries)
  float* sL = reinterpret_cast<float*>(sdS + BN * SP);  // [2][BM] lse * log2e
  float* sD = sL + 2 * BM;                               // [2][BM] delta

  const int kb = blockIdx.x;
  const int bh = blockIdx.y, b = bh / H, h = bh - b * H;
  const int k0 = kb * BN;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, t = lane & 3;
  const long long row_base = static_cast<long long>(b) * S;
  const __nv_bfloat16* qbase = qkv + row_base * ldq + h * 3 * D;
  const __nv_bfloat16* dobase = dout + row_base * lddo + h * D;
  const float* lse_bh = lse + static_cast<long long>(bh) * S;
  const float* delta_bh = delta + static_cast<long long>(bh) * S;

  load_tile<D, DP, BN, 128>(sK, qbase + static_cast<long long>(k0) * ldq + D, ldq, S - k0);
  load_tile<D, DP, BN, 128>(sV, qbase + static_cast<long long>(k0) * ldq + 2 * D, ldq, S - k0);
  const int i_first = k0 / BM;  // causal: queries >= first key of the block
  const int i_last = (S + BM - 1) / BM;
  auto load_q_block = [&](int i, int buf) {
    const int q0 = i * BM;
    load_tile<D, DP, BM, 128>(sQ + buf * BM * DP, qbase + static_cast<long long>(q0) * ldq, ldq, S - q0);
    load_tile<D, DP, BM, 128>(sdO + buf * BM * DP, dobase + static_cast<long long>(q0) * lddo, lddo, S - q0);
    for (int r = threadIdx.x; r < BM; r += 128) {
      const int q = q0 + r;
      sL[buf * BM + r] = q < S ? lse_bh[q] * kLog2e : 0.f;
      sD[buf * BM + r] = q < S ? delta_bh[q] : 0.f;
    }
  };
  load_q_block(i_first, 0);
  cp_async_commit();

  float dk[NT][4], dv[NT][4];
#pragma unroll
  for (int j = 0; j < NT; ++j)
#pragma unroll
    for (int e = 0; e < 4; ++e) dk[j][e] = dv[j][e] = 0.f;

  const int key0 = k0 + warp * 16 + g;  // this thread's keys: key0, key0 + 8

  for (int i = i_first; i < i_last; ++i) {
    const int buf = (i - i_first) & 1;
    if (i + 1 < i_last) {
      load_q_block(i + 1, buf ^ 1);
      cp_async_commit();
      cp_async_wait<1>();
    } else {
      cp_async_wait<0>();
    }
    __syncthreads();
    const __nv_bfloat16* q_s = sQ + buf * BM * DP;
    const __nv_bfloat16* do_s = sdO + buf * BM * DP;
    const float* l_s = sL + buf * BM;
    const float* d_s = sD + buf * BM;
    const int q0 = i * BM;

    // S^T = K_w Q^T and dP^T = V_w dO^T  (16 keys x 64 queries per warp)
    float st[8][4], dpt[8][4];
#pragma unroll
    for (int j = 0; j < 8; ++j)
#pragma unroll
      for (int e = 0; e < 4; ++e) st[j][e] = dpt[j][e] = 0.f;
#pragma unroll
    for (int ks = 0; ks < KS; ++ks) {
      uint32_t ka[4], va[4];
      ldsm_x4(ka, sK + (warp * 16 + (lane & 15)) * DP + ks * 16 + (lane >> 4) * 8);
      ldsm_x4(va, sV + (warp * 16 + (lane & 15)) * DP + ks * 16 + (lane >> 4) * 8);
#pragma unroll
      for (int jp = 0; jp < 4; ++jp) {
        uint32_t qb[4], ob[4];
        const int r = jp * 16 + (lane & 7) + ((lane >> 4) << 3);
        const int c = ks * 16 + ((lane >> 3) & 1) * 8;
        ldsm_x4(qb, q_s + r * DP + c);
        ldsm_x4(ob, do_s + r * DP + c);
        mma16816(st[2 * jp], ka, qb[0], qb[1]);
        mma16816(st[2 * jp + 1], ka, qb[2], qb[3]);
        mma16816(dpt[2 * jp], va, ob[0], ob[1]);
        mma16816(dpt[2 * jp + 1], va, ob[2], ob[3]);
      }
    }
    // P^T = exp(S^T * scale - lse[q]); dS^T = P^T (dP^T - delta[q]).
#pragma unroll
    for (int j = 0; j < 8; ++j) {
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int qc = 8 * j + 2 * t + (e & 1);
        const int q = q0 + qc;
        const int key = key0 + ((e >> 1) << 3);
        float p = ex2(st[j][e] * scale_log2 - l_s[qc]);
        if (key > q || q >= S || key >= S) p = 0.f;
        st[j][e] = p;
        dpt[j][e] = p * (dpt[j][e] - d_s[qc]);
      }
    }
    // dV += P^T dO ; dK += dS^T Q   (contraction over the 64 queries)
#pragma unroll
    for (int kk = 0; kk < 4; ++kk) {
      uint32_t pa[4], sa[4];
      pa[0] = pack_bf16x2(st[2 * kk][0], st[2 * kk][1]);
      pa[1] = pack_bf16x2(st[2 * kk][2], st[2 * kk][3]);
      pa[2] = pack_bf16x2(st[2 * kk + 1][0], st[2 * kk + 1][1]);
      pa[3] = pack_bf16x2(st[2 * kk + 1][2], st[2 * kk + 1][3]);
      sa[0] = pack_bf16x2(dpt[2 * kk][0], dpt[2 * kk][1]);
      sa[1] = pack_bf16x2(dpt[2 * kk][2], dpt[2 * kk][3]);
      sa[2] = pack_bf16x2(dpt[2 * kk + 1][0], dpt[2 * kk + 1][1]);
      sa[3] = pack_bf16x2(dpt[2 * kk + 1][2], dpt[2 * kk + 1][3]);
#pragma unroll
      for (int jp = 0; jp < NT / 2; ++jp) {
        uint32_t ob[4], qb[4];
        const int r = kk * 16 + (lane & 7) + (((lane >> 3) & 1) << 3);
        const int c = jp * 16 + (lane >> 4) * 8;
        ldsm_x4_t(ob, do_s + r * DP + c);
        ldsm_x4_t(qb, q_s + r * DP + c);
        mma16816(dv[2 * jp], pa, ob[0], ob[1]);
        mma16816(dv[2 * jp + 1], pa, ob[2], ob[3]);
        mma16816(dk[2 * jp], sa, qb[0], qb[1]);
        mma16816(dk[2 * jp + 1], sa, qb[2], qb[3]);
      }
      // Stage dS^T for the dQ product.
      const int kr = warp * 16 + g;
      *reinterpret_cast<uint32_t*>(sdS + kr * SP + 16 * kk + 2 * t) = sa[0];
      *reinterpret_cast<uint32_t*>(sdS + (kr + 8) * SP + 16 * kk + 2 * t) = sa[1];
      *reinterpret_cast<uint32_t*>(sdS + kr * SP + 16 * kk + 8 + 2 * t) = sa[2];
      *reinterpret_cast<uint32_t*>(sdS + (kr + 8) * SP + 16 * kk + 8 + 2 * t) = sa[3];
    }
    __syncthreads();
    // dQ[16 queries of this warp] += dS K  (contraction over the 64 keys).
    uint32_t da[4][4];
#pragma unroll
    for (int kk = 0; kk < 4; ++kk)
      ldsm_x4_t(da[kk], sdS + (kk * 16 + (lane & 7) + ((lane >> 4) << 3)) * SP + warp * 16 + ((lane >> 3) & 1) * 8);
    const int qa = q0 + warp * 16 + g, qb2 = qa + 8;
#pragma unroll
    for (int jp = 0; jp < NT / 2; ++jp) {
      float acc[2][4];
#pragma unroll
      for (int e = 0; e < 4; ++e) acc[0][e] = acc[1][e] = 0.f;
#pragma unroll
      for (int kk = 0; kk < 4; ++kk) {
        uint32_t kbf[4];
        ldsm_x4_t(kbf, sK + (kk * 16 + (lane & 7) + (((lane >> 3) & 1) << 3)) * DP + jp * 16 + (lane >> 4) * 8);
        mma16816(acc[0], da[kk], kbf[0], kbf[1]);
        mma16816(acc[1], da[kk], kbf[2], kbf[3]);
      }
#pragma unroll
      for (int u = 0; u < 2; ++u) {
        const int col = h * D + jp * 16 + u * 8 + 2 * t;
        if (qa < S) red_add_f32x2(dqacc + (row_base + qa) * ldacc + col, acc[u][0], acc[u][1]);
        if (qb2 < S) red_add_f32x2(dqacc + (row_base + qb2) * ldacc + col, acc[u][2], acc[u][3]);
      }
    }
    __syncthreads();  // sdS and this Q/dO buffer are rewritten next iteration
  }

  // dK (scaled) and dV for this warp's 16 keys.
  const int kr0 = key0, kr1 = key0 + 8;
#pragma unroll
  for (int j = 0; j < NT; ++j) {
    const int col = h * 3 * D + 8 * j + 2 * t;
    if (kr0 < S) {
      __nv_bfloat16* r = dqkv + (row_base + kr0) * lddq + col;
      *reinterpret_cast<uint32_t*>(r + D) = pack_bf16x2(dk[j][0] * scale, dk[j][1] * scale);
      *reinterpret_cast<uint32_t*>(r + 2 * D) = pack_bf16x2(dv[j][0], dv[j][1]);
    }
    if (kr1 < S) {
      __nv_bfloat16* r = dqkv + (row_base + kr1) * lddq + col;
      *reinterpret_cast<uint32_t*>(r + D) = pack_bf16x2(dk[j][2] * scale, dk[j][3] * scale);
      *reinterpret_cast<uint32_t*>(r + 2 * D) = pack_bf16x2(dv[j][2], dv[j][3]);
    }
  }
}

}  // namespace attn
}  // namespace md

// ============================================================================
// Host entry points
// ============================================================================
namespace {

template <int D>
size_t fwd_smem() { return static_cast<size_t>(128 + 4 * 64) * (D + 8) * 2; }
template <int D>
size_t bwd_smem() { return static_cast<size_t>(6 * 64) * (D + 8) * 2 + 64 * 72 * 2 + 4 * 64 * 4; }

template <int D>
int fwd_launch(const void* qkv, long long ldq, void* out, long long ldo, float* lse, int B, int H, int S,
               float scale, cudaStream_t st) {
  auto k = md::attn::fwd_kernel<D>;
  const size_t smem = fwd_smem<D>();
  cudaError_t e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
  if (e != cudaSuccess) return static_cast<int>(e);
  dim3 grid((S + 127) / 128, B * H);
  md::launch_pdl(k, dim3(grid), dim3(256), smem, st, reinterpret_cast<const __nv_bfloat16*>(qkv), ldq, reinterpret_cast<__nv_bfloat16*>(out),
      ldo, lse, H, S, scale * md::attn::kLog2e);
  return static_cast<int>(cudaGetLastError());
}

template <int D>
int bwd_launch(const void* qkv, long long ldq, const void* out, long long ldo, const void* dout, long long lddo,
               const float* lse, float* delta, float* dqacc, void* dqkv, long long lddq, int B, int H, int S,
               float scale, cudaStream_t st) {
  const long long rows = static_cast<long long>(B) * S;
  cudaError_t e = cudaMemsetAsync(dqacc, 0, rows * H * D * sizeof(float), st);
  if (e != cudaSuccess) return static_cast<int>(e);
  const long long nd = static_cast<long long>(B) * H * S;
  int g1 = static_cast<int>((nd + 255) / 256);
  if (g1 > 148 * 32) g1 = 148 * 32;
  md::launch_pdl(md::attn::delta_kernel<D>, dim3(g1), dim3(256), 0, st, reinterpret_cast<const __nv_bfloat16*>(out), ldo,
      reinterpret_cast<const __nv_bfloat16*>(dout), lddo, delta, B, H, S);
  auto k = md::attn::bwd_kernel<D>;
  const size_t smem = bwd_smem<D>();
  e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
  if (e != cudaSuccess) return static_cast<int>(e);
  dim3 grid((S + 63) / 64, B * H);
  md::launch_pdl(k, dim3(grid), dim3(128), smem, st, reinterpret_cast<const __nv_bfloat16*>(qkv), ldq,
      reinterpret_cast<const __nv_bfloat16*>(dout), lddo, lse, delta, dqacc,
      static_cast<long long>(H) * D, reinterpret_cast<__nv_bfloat16*>(dqkv), lddq, H, S, scale,
      scale * md::attn::kLog2e);
  const long long nq = rows * H * (D / 2);
  int g2 = static_cast<int>((nq + 255) / 256);
  if (g2 > 148 * 32) g2 = 148 * 32;
  md::launch_pdl(md::attn::dq_convert_kernel<D>, dim3(g2), dim3(256), 0, st, dqacc, static_cast<long long>(H) * D,
      reinterpret_cast<__nv_bfloat16*>(dqkv), lddq,
      static_cast<int>(rows), H, scale);
  return static_cast<int>(cudaGetLastError());
}

bool al16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

}  // namespace

extern "C" {

// qkv: [B*S, ldq] bf16 with per-head interleaved [H, 3, D] columns; out: [B*S, ldo]
// (head h at columns h*D); lse: [B, H, S] fp32.
int md_attn_fwd(const void* qkv, long long ldq, void* out, long long ldo, float* lse, int B, int H, int S, int D,
                float scale, cudaStream_t st) {
  if (B <= 0 || H <= 0 || S <= 0 || !al16(qkv) || !al16(out) || (ldq % 8) || (ldo % 8)) return -1;
  switch (D) {
    case 32: return fwd_launch<32>(qkv, ldq, out, ldo, lse, B, H, S, scale, st);
    case 64: return fwd_launch<64>(qkv, ldq, out, ldo, lse, B, H, S, scale, st);
    case 80: return fwd_launch<80>(qkv, ldq, out, ldo, lse, B, H, S, scale, st);
    case 128: return fwd_launch<128>(qkv, ldq, out, ldo, lse, B, H, S, scale, st);
    default: return -2;
  }
}

// Scratch: delta [B*H*S] fp32 and dqacc [B*S, H*D] fp32 (zeroed here).
// dqkv receives dQ/dK/dV in the same interleaved layout as qkv.
int md_attn_bwd(const void* qkv, long long ldq, const void* out, long long ldo, const void* dout, long long lddo,
                const float* lse, float* delta, float* dqacc, void* dqkv, long long lddq, int B, int H, int S, int D,
                float scale, cudaStream_t st) {
  if (B <= 0 || H <= 0 || S <= 0 || !al16(qkv) || !al16(out) || !al16(dout) || !al16(dqkv) || (ldq % 8) ||
      (ldo % 8) || (lddo % 8) || (lddq % 8))
    return -1;
  switch (D) {
    case 32: return bwd_launch<32>(qkv, ldq, out, ldo, dout, lddo, lse, delta, dqacc, dqkv, lddq, B, H, S, scale, st);
    case 64: return bwd_launch<64>(qkv, ldq, out, ldo, dout, lddo, lse, delta, dqacc, dqkv, lddq, B, H, S, scale, st);
    case 80: return bwd_launch<80>(qkv, ldq, out, ldo, dout, lddo, lse, delta, dqacc, dqkv, lddq, B, H, S, scale, st);
    case 128:
      return bwd_launch<128>(qkv, ldq, out, ldo, dout, lddo, lse, delta, dqacc, dqkv, lddq, B, H, S, scale, st);
    default: return -2;
  }
}

// Backward through the tcgen05 main kernel of attention_sm100.cu (head_dim
// 64): same contract as md_attn_bwd, plus the status word for timed-out waits.
int md_attn_bwd_tc_main(const void* qkv, long long ldq, const void* dout, long long lddo, const float* lse,
                        const float* delta, float* dqacc, long long ldacc, void* dqkv, long long lddq, int B, int H,
                        int S, int D, float scale, void* status, cudaStream_t st);

int md_attn_bwd_tc(const void* qkv, long long ldq, const void* out, long long ldo, const void* dout, long long lddo,
                   const float* lse, float* delta, float* dqacc, void* dqkv, long long lddq, int B, int H, int S,
                   int D, float scale, void* status, cudaStream_t st) {
  if (B <= 0 || H <= 0 || S <= 0 || !al16(qkv) || !al16(out) || !al16(dout) || !al16(dqkv) || (ldq % 8) ||
      (ldo % 8) || (lddo % 8) || (lddq % 8))
    return -1;
  if (D != 64 && D != 80 && D != 128) return -2;
  const long long rows = static_cast<long long>(B) * S;
  cudaError_t e = cudaMemsetAsync(dqacc, 0, rows * H * D * sizeof(float), st);
  if (e != cudaSuccess) return static_cast<int>(e);
  const long long nd = static_cast<long long>(B) * H * S;
  int g1 = static_cast<int>((nd + 255) / 256);
  if (g1 > 148 * 32) g1 = 148 * 32;
  // out == null: delta was produced upstream (the epilogue of the GEMM that made dout).
  if (out != nullptr) {
    const __nv_bfloat16* o = reinterpret_cast<const __nv_bfloat16*>(out);
    const __nv_bfloat16* d = reinterpret_cast<const __nv_bfloat16*>(dout);
    if (D == 64) md::launch_pdl(md::attn::delta_kernel<64>, dim3(g1), dim3(256), 0, st, o, ldo, d, lddo, delta, B, H, S);
    if (D == 80) md::launch_pdl(md::attn::delta_kernel<80>, dim3(g1), dim3(256), 0, st, o, ldo, d, lddo, delta, B, H, S);
    if (D == 128) md::launch_pdl(md::attn::delta_kernel<128>, dim3(g1), dim3(256), 0, st, o, ldo, d, lddo, delta, B, H, S);
  }
  int rc = md_attn_bwd_tc_main(qkv, ldq, dout, lddo, lse, delta, dqacc, static_cast<long long>(H) * D, dqkv, lddq, B,
                               H, S, D, scale, status, st);
  if (rc != 0) return rc;
  const long long nq = rows * H * (D / 8);
  int g2 = static_cast<int>((nq + 255) / 256);
  if (g2 > 148 * 32) g2 = 148 * 32;
  __nv_bfloat16* dq = reinterpret_cast<__nv_bfloat16*>(dqkv);
  const long long lda = static_cast<long long>(H) * D;
  if (D == 64)
    md::launch_pdl(md::attn::dq_convert_kernel<64>, dim3(g2), dim3(256), 0, st, dqacc, lda, dq, lddq, static_cast<int>(rows), H, scale);
  if (D == 80)
    md::launch_pdl(md::attn::dq_convert_kernel<80>, dim3(g2), dim3(256), 0, st, dqacc, lda, dq, lddq, static_cast<int>(rows), H, scale);
  if (D == 128)
    md::launch_pdl(md::attn::dq_convert_kernel<128>, dim3(g2), dim3(256), 0, st, dqacc, lda, dq, lddq, static_cast<int>(rows), H, scale);
  return static_cast<int>(cudaGetLastError());
}

}  // extern "C"
