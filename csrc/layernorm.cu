// LayerNorm forward/backward for bf16 activations with fp32 statistics and
// fp32 affine parameters (the model keeps fp32 master weights).
//
// A row of C elements (C % 8 == 0) is handled by a "team" of T threads; every
// thread holds up to V 16-byte vectors (8 bf16 each) in registers, so the row
// is read once.  T scales with C so the per-thread footprint stays at <= 32
// values: T=32 up to C=1024, 64 up to 2048, 128 up to 4096, 256 up to 8192.
//
// Backward accumulates dgamma/dbeta per thread over the rows its team
// processes, then reduces across teams in shared memory in a fixed order and
// writes one partial row per CTA; md_ln_reduce_partials sums the CTA partials
// in a fixed order too.  The result is bit-reproducible, which keeps
// LayerNorm gradients of tensor-parallel replicas identical on every rank.
//
// The backward optionally fuses two column sums the transformer block needs
// anyway (the bias gradients of the row-parallel projections on either side of
// the norm): the column sum of the incoming residual gradient and of the
// produced input gradient.
//
// Replaces nn.LayerNorm (reference models/gpt.py:158,160,199) and the ATen
// layer_norm kernels it dispatches to.
#include "md_sm100.cuh"

namespace md {
namespace ln {

constexpr int kThreads = 256;

template <int T>
__device__ __forceinline__ float team_sum(float v, float* scratch) {
  // scratch: [kThreads / 32] floats per CTA (used only when T > 32)
#pragma unroll
  for (int o = (T < 32 ? T : 32) / 2; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  if constexpr (T > 32) {
    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const int team_first_warp = (threadIdx.x / T) * (T / 32);
    __syncwarp();
    if (lane == 0) scratch[warp] = v;
    // All warps of a team must publish before any reads.  Teams are aligned to
    // warps, so a named barrier per team is not needed: the whole CTA syncs.
    __syncthreads();
    float s = 0.f;
#pragma unroll
    for (int w = 0; w < T / 32; ++w) s += scratch[team_first_warp + w];
    __syncthreads();
    v = s;
  }
  return v;
}

template <int T, int V>
__global__ void __launch_bounds__(kThreads) ln_fwd_kernel(const __nv_bfloat16* __restrict__ x, long long ldx,
                                                         const float* __restrict__ gamma,
                                                         const float* __restrict__ beta,
                                                         __nv_bfloat16* __restrict__ y, long long ldy,
                                                         float* __restrict__ mean_out, float* __restrict__ rstd_out,
                                                         int M, int C, float eps) {
  pdl_trigger();  // the next kernel may launch now
  pdl_wait();     // global memory only after the previous kernel completed
  __shared__ float scratch[kThreads / 32];
  const int teams_per_cta = kThreads / T;
  const int team = threadIdx.x / T;
  const int t = threadIdx.x % T;
  const int nvec = C / 8;
  const float inv_c = 1.0f / static_cast<float>(C);
  // Every team runs the same number of iterations so the CTA-wide barriers in
  // team_sum (T > 32) line up; rows past M are computed on a clamped row and
  // not stored.
  const int rows_per_pass = gridDim.x * teams_per_cta;
  const int passes = (M + rows_per_pass - 1) / rows_per_pass;
  for (int pass = 0; pass < passes; ++pass) {
    const int row = pass * rows_per_pass + blockIdx.x * teams_per_cta + team;
    const bool valid = row < M;
    const int r = valid ? row : M - 1;
    float v[V][8];
    float s = 0.f;
#pragma unroll
    for (int i = 0; i < V; ++i) {
      const int j = t + i * T;
      if (j < nvec) {
        uint4 w = reinterpret_cast<const uint4*>(x + r * ldx)[j];
        float2 a = unpack_bf16x2(w.x), b = unpack_bf16x2(w.y), c = unpack_bf16x2(w.z), d = unpack_bf16x2(w.w);
        v[i][0] = a.x; v[i][1] = a.y; v[i][2] = b.x; v[i][3] = b.y;
        v[i][4] = c.x; v[i][5] = c.y; v[i][6] = d.x; v[i][7] = d.y;
#pragma unroll
        for (int e = 0; e < 8; ++e) s += v[i][e];
      }
    }
    const float mean = team_sum<T>(s, scratch) * inv_c;
    float q = 0.f;
#pragma unroll
    for (int i = 0; i < V; ++i) {
      const int j = t + i * T;
      if (j < nvec) {
#pragma unroll
        for (int e = 0; e < 8; ++e) {
          const float d = v[i][e] - mean;
          q += d * d;
        }
      }
    }
    const float rstd = rsqrtf(team_sum<T>(q, scratch) * inv_c + eps);
    if (!valid) continue;
#pragma unroll
    for (int i = 0; i < V; ++i) {
      const int j = t + i * T;
      if (j < nvec) {
        const float4 g0 = reinterpret_cast<const float4*>(gamma)[2 * j];
        const float4 g1 = reinterpret_cast<const float4*>(gamma)[2 * j + 1];
        const float4 b0 = reinterpret_cast<const float4*>(beta)[2 * j];
        const float4 b1 = reinterpret_cast<const float4*>(beta)[2 * j + 1];
        const float g[8] = {g0.x, g0.y, g0.z, g0.w, g1.x, g1.y, g1.z, g1.w};
        const float b[8] = {b0.x, b0.y, b0.z, b0.w, b1.x, b1.y, b1.z, b1.w};
        float o[8];
#pragma unroll
        for (int e = 0; e < 8; ++e) o[e] = (v[i][e] - mean) * rstd * g[e] + b[e];
        uint4 w;
        w.x = pack_bf16x2(o[0], o[1]);
        w.y = pack_bf16x2(o[2], o[3]);
        w.z = pack_bf16x2(o[4], o[5]);
        w.w = pack_bf16x2(o[6], o[7]);
        reinterpret_cast<uint4*>(y + row * ldy)[j] = w;
      }
    }
    if (t == 0) {
      mean_out[row] = mean;
      rstd_out[row] = rstd;
    }
  }
}

// NACC = 2 (dgamma, dbeta) or 4 (+ colsum(resid_grad), colsum(dx)).
template <int T, int V, int NACC>
__global__ void __launch_bounds__(kThreads) ln_bwd_kernel(
    const __nv_bfloat16* __restrict__ dy, long long lddy, const __nv_bfloat16* __restrict__ x, long long ldx,
    const float* __restrict__ mean_in, const float* __restrict__ rstd_in, const float* __restrict__ gamma,
    const __nv_bfloat16* __restrict__ resid_grad, long long ldr, __nv_bfloat16* __restrict__ dx, long long lddx,
    float* __restrict__ partials, int M, int C) {
  pdl_trigger();  // the next kernel may launch now
  pdl_wait();     // global memory only after the previous kernel completed
  extern __shared__ float smem_f[];  // [teams][NACC][C] then scratch
  const int teams_per_cta = kThreads / T;
  const int team = threadIdx.x / T;
  const int t = threadIdx.x % T;
  const int nvec = C / 8;
  const float inv_c = 1.0f / static_cast<float>(C);
  float* scratch = smem_f + teams_per_cta * NACC * C;

  float acc[NACC][V][8];
#pragma unroll
  for (int a = 0; a < NACC; ++a)
#pragma unroll
    for (int i = 0; i < V; ++i)
#pragma unroll
      for (int e = 0; e < 8; ++e) acc[a][i][e] = 0.f;

  const int rows_per_pass = gridDim.x * teams_per_cta;
  const int passes = (M + rows_per_pass - 1) / rows_per_pass;
  for (int pass = 0; pass < passes; ++pass) {
    const int row = pass * rows_per_pass + blockIdx.x * teams_per_cta + team;
    const bool valid = row < M;
    const int r = valid ? row : M - 1;
    const float mean = mean_in[r], rstd = rstd_in[r];
    float xh[V][8], gy[V][8];
    float s1 = 0.f, s2 = 0.f;
#pragma unroll
    for (int i = 0; i < V; ++i) {
      const int j = t + i * T;
      if (j < nvec) {
        uint4 wx = reinterpret_cast<const uint4*>(x + r * ldx)[j];
        uint4 wd = reinterpret_cast<const uint4*>(dy + r * lddy)[j];
        const float4 g0 = reinterpret_cast<const float4*>(gamma)[2 * j];
        const float4 g1 = reinterpret_cast<const float4*>(gamma)[2 * j + 1];
        const float g[8] = {g0.x, g0.y, g0.z, g0.w, g1.x, g1.y, g1.z, g1.w};
        const uint32_t xs[4] = {wx.x, wx.y, wx.z, wx.w};
        const uint32_t ds[4] = {wd.x, wd.y, wd.z, wd.w};
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const float2 xv = unpack_bf16x2(xs[q]);
          const float2 dv = unpack_bf16x2(ds[q]);
          xh[i][2 * q] = (xv.x - mean) * rstd;
          xh[i][2 * q + 1] = (xv.y - mean) * rstd;
          if (valid) {
            acc[0][i][2 * q] += dv.x * xh[i][2 * q];
            acc[0][i][2 * q + 1] += dv.y * xh[i][2 * q + 1];
            acc[1][i][2 * q] += dv.x;
            acc[1][i][2 * q + 1] += dv.y;
          }
          gy[i][2 * q] = dv.x * g[2 * q];
          gy[i][2 * q + 1] = dv.y * g[2 * q + 1];
        }
#pragma unroll
        for (int e = 0; e < 8; ++e) {
          s1 += gy[i][e];
          s2 += gy[i][e] * xh[i][e];
        }
      }
    }
    const float a1 = team_sum<T>(s1, scratch) * inv_c;
    const float a2 = team_sum<T>(s2, scratch) * inv_c;
    if (!valid) continue;
#pragma unroll
    for (int i = 0; i < V; ++i) {
      const int j = t + i * T;
      if (j < nvec) {
        float o[8];
#pragma unroll
        for (int e = 0; e < 8; ++e) o[e] = rstd * (gy[i][e] - a1 - xh[i][e] * a2);
        if (resid_grad != nullptr) {
          uint4 wr = reinterpret_cast<const uint4*>(resid_grad + row * ldr)[j];
          const uint32_t rs[4] = {wr.x, wr.y, wr.z, wr.w};
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            const float2 rv = unpack_bf16x2(rs[q]);
            o[2 * q] += rv.x;
            o[2 * q + 1] += rv.y;
            if constexpr (NACC == 4) {
              acc[2][i][2 * q] += rv.x;
              acc[2][i][2 * q + 1] += rv.y;
            }
          }
        }
        uint4 w;
        w.x = pack_bf16x2(o[0], o[1]);
        w.y = pack_bf16x2(o[2], o[3]);
        w.z = pack_bf16x2(o[4], o[5]);
        w.w = pack_bf16x2(o[6], o[7]);
        reinterpret_cast<uint4*>(dx + row * lddx)[j] = w;
        if constexpr (NACC == 4) {
          // Column sum of the *stored* (bf16-rounded) gradient, as the next
          // GEMM will see it.
          const uint32_t ws[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            const float2 ov = unpack_bf16x2(ws[q]);
            acc[3][i][2 * q] += ov.x;
            acc[3][i][2 * q + 1] += ov.y;
          }
        }
      }
    }
  }

  // Fixed-order cross-team reduction, then one partial row per CTA.
#pragma unroll
  for (int a = 0; a < NACC; ++a)
#pragma unroll
    for (int i = 0; i < V; ++i) {
      const int j = t + i * T;
      if (j < nvec)
#pragma unroll
        for (int e = 0; e < 8; ++e) smem_f[(team * NACC + a) * C + j * 8 + e] = acc[a][i][e];
    }
  __syncthreads();
  for (int idx = threadIdx.x; idx < NACC * C; idx += kThreads) {
    float s = 0.f;
    for (int tm = 0; tm < teams_per_cta; ++tm) s += smem_f[tm * NACC * C + idx];
    partials[static_cast<long long>(blockIdx.x) * NACC * C + idx] = s;
  }
}

// Backward for rows of up to 1024 columns (one warp per row, lane l owns the
// 16-byte vectors j = l + 32 i).  Same math and outputs as ln_bwd_kernel, but
// every lane streams its own vectors of dy, x and resid_grad through a
// kStages-deep cp.async ring in shared memory, so each warp has the next
// kStages-1 rows in flight while it computes the current one (the register
// version held one row per warp in flight: ~30 % of DRAM bandwidth).  A lane
// reads back only what it copied itself, so no cross-lane synchronisation is
// needed until the final fixed-order reduction, which reuses the ring.
constexpr int kPipeStages = 4;
// Backward ring: three stages, so that at C <= 768 (V <= 3) two CTAs fit on
// an SM (2 x 111 KB): 16 warps instead of 8 hide the load and shuffle
// latency of the per-row reductions.  (Only with two accumulators -- dgamma,
// dbeta -- does a thread fit the 128 registers two CTAs allow; the variant
// that also sums two more columns keeps one CTA per SM.)
template <int V, int NACC>
__host__ __device__ constexpr int bwd_stages() { return (NACC == 2 && V <= 3) ? 3 : 4; }

__device__ __forceinline__ void cp_async16_ln(uint32_t smem, const void* gmem) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem), "l"(gmem) : "memory");
}
__device__ __forceinline__ void cp_async_commit_ln() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait_ln() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

// Forward for rows of up to 1024 columns with the same per-lane cp.async ring
// (kPipeStages - 1 rows in flight per warp): mean and variance in two passes
// over registers, gamma and beta held in registers for the whole kernel.
template <int V>
__global__ void __launch_bounds__(kThreads, 2) ln_fwd_pipe_kernel(const __nv_bfloat16* __restrict__ x, long long ldx,
                                                              const float* __restrict__ gamma,
                                                              const float* __restrict__ beta,
                                                              __nv_bfloat16* __restrict__ y, long long ldy,
                                                              float* __restrict__ mean_out, float* __restrict__ rstd_out,
                                                              int M, int C, float eps) {
  pdl_trigger();  // the next kernel may launch now
  pdl_wait();     // global memory only after the previous kernel completed
  extern __shared__ __align__(16) uint8_t smem_u8[];
  constexpr int kWarps = kThreads / 32;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nvec = C / 8;
  const float inv_c = 1.0f / static_cast<float>(C);
  uint8_t* ring = smem_u8 + static_cast<size_t>(warp) * kPipeStages * V * 32 * 16;
  auto slot = [&](int st, int i) -> uint32_t { return smem_u32(ring + ((st * V + i) * 32 + lane) * 16); };
  const int rows_per_pass = gridDim.x * kWarps;
  const int first = blockIdx.x * kWarps + warp;
  const int passes = first < M ? (M - 1 - first) / rows_per_pass + 1 : 0;
  auto issue = [&](int pass) {
    if (pass < passes) {
      const long long r = first + static_cast<long long>(pass) * rows_per_pass;
#pragma unroll
      for (int i = 0; i < V; ++i) {
        const int j = lane + 32 * i;
        if (j < nvec) cp_async16_ln(slot(pass % kPipeStages, i), reinterpret_cast<const uint4*>(x + r * ldx) + j);
      }
    }
    cp_async_commit_ln();
  };
  float gam[V][8], bet[V][8];
#pragma unroll
  for (int i = 0; i < V; ++i) {
    const int j = lane + 32 * i;
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      gam[i][e] = j < nvec ? gamma[8 * j + e] : 0.f;
      bet[i][e] = j < nvec ? beta[8 * j + e] : 0.f;
    }
  }
#pragma unroll
  for (int k = 0; k < kPipeStages - 1; ++k) issue(k);
  for (int pass = 0; pass < passes; ++pass) {
    issue(pass + kPipeStages - 1);
    cp_async_wait_ln<kPipeStages - 1>();
    const long long row = first + static_cast<long long>(pass) * rows_per_pass;
    const int st = pass % kPipeStages;
    float v[V][8];
    float s = 0.f;
#pragma unroll
    for (int i = 0; i < V; ++i) {
      const int j = lane + 32 * i;
      if (j < nvec) {
        uint4 w;
        asm volatile("ld.shared.v4.b32 {%0, %1, %2, %3}, [%4];" : "=r"(w.x), "=r"(w.y), "=r"(w.z), "=r"(w.w)
                     : "r"(slot(st, i)));
        const uint32_t ws[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const float2 f = unpack_bf16x2(ws[q]);
          v[i][2 * q] = f.x;
          v[i][2 * q + 1] = f.y;
          s += f.x + f.y;
        }
      } else {
#pragma unroll
        for (int e = 0; e < 8; ++e) v[i][e] = 0.f;
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
    const float mean = s * inv_c;
    float q2 = 0.f;
#pragma unroll
    for (int i = 0; i < V; ++i) {
      const int j = lane + 32 * i;
      if (j < nvec)
#pragma unroll
        for (int e = 0; e < 8; ++e) {
          const float d = v[i][e] - mean;
          q2 += d * d;
        }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) q2 += __shfl_xor_sync(0xffffffffu, q2, o);
    const float rstd = rsqrtf(q2 * inv_c + eps);
#pragma unroll
    for (int i = 0; i < V; ++i) {
      const int j = lane + 32 * i;
      if (j < nvec) {
        float o[8];
#pragma unroll
        for (int e = 0; e < 8; ++e) o[e] = (v[i][e] - mean) * rstd * gam[i][e] + bet[i][e];
        uint4 w;
        w.x = pack_bf16x2(o[0], o[1]);
        w.y = pack_bf16x2(o[2], o[3]);
        w.z = pack_bf16x2(o[4], o[5]);
        w.w = pack_bf16x2(o[6], o[7]);
        reinterpret_cast<uint4*>(y + row * ldy)[j] = w;
      }
    }
    if (lane == 0) {
      mean_out[row] = mean;
      rstd_out[row] = rstd;
    }
  }
  cp_async_wait_ln<0>();
}

template <int V, int NACC>
__global__ void __launch_bounds__(kThreads, (NACC == 2 && V <= 3) ? 2 : 1) ln_bwd_pipe_kernel(
    const __nv_bfloat16* __restrict__ dy, long long lddy, const __nv_bfloat16* __restrict__ x, long long ldx,
    const float* __restrict__ mean_in, const float* __restrict__ rstd_in, const float* __restrict__ gamma,
    const __nv_bfloat16* __restrict__ resid_grad, long long ldr, __nv_bfloat16* __restrict__ dx, long long lddx,
    float* __restrict__ partials, int M, int C) {
  constexpr int kBwdStages = bwd_stages<V, NACC>();
  pdl_trigger();  // the next kernel may launch now
  pdl_wait();     // global memory only after the previous kernel completed
  extern __shared__ __align__(16) uint8_t smem_u8[];
  constexpr int kWarps = kThreads / 32;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nvec = C / 8;
  const float inv_c = 1.0f / static_cast<float>(C);
  const bool has_r = resid_grad != nullptr;
  // Ring: [warp][stage][tensor (dy, x, r)][V][32 lanes] x 16 bytes, then
  // [warp][stage] x (mean, rstd) copied by lane 0.
  uint8_t* ring = smem_u8 + static_cast<size_t>(warp) * kBwdStages * 3 * V * 32 * 16;
  float* stats = reinterpret_cast<float*>(smem_u8 + static_cast<size_t>(kWarps) * kBwdStages * 3 * V * 32 * 16) +
                 warp * kBwdStages * 2;
  auto slot = [&](int st, int tsr, int i) -> uint32_t {
    return smem_u32(ring + (((st * 3 + tsr) * V + i) * 32 + lane) * 16);
  };
  const int rows_per_pass = gridDim.x * kWarps;
  const int first = blockIdx.x * kWarps + warp;
  const int passes = first < M ? (M - 1 - first) / rows_per_pass + 1 : 0;
  auto issue = [&](int pass) {
    if (pass < passes) {
      const long long r = first + static_cast<long long>(pass) * rows_per_pass;
      const int st = pass % kBwdStages;
#pragma unroll
      for (int i = 0; i < V; ++i) {
        const int j = lane + 32 * i;
        if (j < nvec) {
          cp_async16_ln(slot(st, 0, i), reinterpret_cast<const uint4*>(dy + r * lddy) + j);
          cp_async16_ln(slot(st, 1, i), reinterpret_cast<const uint4*>(x + r * ldx) + j);
          if (has_r) cp_async16_ln(slot(st, 2, i), reinterpret_cast<const uint4*>(resid_grad + r * ldr) + j);
        }
      }
      if (lane == 0) {
        asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(smem_u32(stats + 2 * st)), "l"(mean_in + r)
                     : "memory");
        asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(smem_u32(stats + 2 * st + 1)), "l"(rstd_in + r)
                     : "memory");
      }
    }
    cp_async_commit_ln();  // empty groups keep the count uniform
  };

  float acc[NACC][V][8];
#pragma unroll
  for (int a = 0; a < NACC; ++a)
#pragma unroll
    for (int i = 0; i < V; ++i)
#pragma unroll
      for (int e = 0; e < 8; ++e) acc[a][i][e] = 0.f;
  float gam[V][8];
#pragma unroll
  for (int i = 0; i < V; ++i) {
    const int j = lane + 32 * i;
#pragma unroll
    for (int e = 0; e < 8; ++e) gam[i][e] = j < nvec ? gamma[8 * j + e] : 0.f;
  }

#pragma unroll
  for (int k = 0; k < kBwdStages - 1; ++k) issue(k);
  for (int pass = 0; pass < passes; ++pass) {
    __syncwarp();  // every lane has read the previous row's statistics before lane 0 refills that slot
    issue(pass + kBwdStages - 1);
    cp_async_wait_ln<kBwdStages - 1>();
    __syncwarp();  // lane 0's statistics copy is visible to the warp
    const long long row = first + static_cast<long long>(pass) * rows_per_pass;
    const int st = pass % kBwdStages;
    const float mean = stats[2 * st], rstd = stats[2 * st + 1];
    float s1 = 0.f, s2 = 0.f;
#pragma unroll
    for (int i = 0; i < V; ++i) {
      const int j = lane + 32 * i;
      if (j < nvec) {
        uint4 wd, wx;
        asm volatile("ld.shared.v4.b32 {%0, %1, %2, %3}, [%4];" : "=r"(wd.x), "=r"(wd.y), "=r"(wd.z), "=r"(wd.w)
                     : "r"(slot(st, 0, i)));
        asm volatile("ld.shared.v4.b32 {%0, %1, %2, %3}, [%4];" : "=r"(wx.x), "=r"(wx.y), "=r"(wx.z), "=r"(wx.w)
                     : "r"(slot(st, 1, i)));
        const uint32_t ds[4] = {wd.x, wd.y, wd.z, wd.w}, xs[4] = {wx.x, wx.y, wx.z, wx.w};
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const float2 dv = unpack_bf16x2(ds[q]), xv = unpack_bf16x2(xs[q]);
          const float h0 = (xv.x - mean) * rstd, h1 = (xv.y - mean) * rstd;
          acc[0][i][2 * q] += dv.x * h0;
          acc[0][i][2 * q + 1] += dv.y * h1;
          acc[1][i][2 * q] += dv.x;
          acc[1][i][2 * q + 1] += dv.y;
          const float g0 = dv.x * gam[i][2 * q], g1 = dv.y * gam[i][2 * q + 1];
          s1 += g0 + g1;
          s2 += g0 * h0 + g1 * h1;
        }
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      s1 += __shfl_xor_sync(0xffffffffu, s1, o);
      s2 += __shfl_xor_sync(0xffffffffu, s2, o);
    }
    const float a1 = s1 * inv_c, a2 = s2 * inv_c;
#pragma unroll
    for (int i = 0; i < V; ++i) {
      const int j = lane + 32 * i;
      if (j < nvec) {
        uint4 wd, wx;
        asm volatile("ld.shared.v4.b32 {%0, %1, %2, %3}, [%4];" : "=r"(wd.x), "=r"(wd.y), "=r"(wd.z), "=r"(wd.w)
                     : "r"(slot(st, 0, i)));
        asm volatile("ld.shared.v4.b32 {%0, %1, %2, %3}, [%4];" : "=r"(wx.x), "=r"(wx.y), "=r"(wx.z), "=r"(wx.w)
                     : "r"(slot(st, 1, i)));
        const uint32_t ds[4] = {wd.x, wd.y, wd.z, wd.w}, xs[4] = {wx.x, wx.y, wx.z, wx.w};
        float o[8];
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const float2 dv = unpack_bf16x2(ds[q]), xv = unpack_bf16x2(xs[q]);
          o[2 * q] = rstd * (dv.x * gam[i][2 * q] - a1 - (xv.x - mean) * rstd * a2);
          o[2 * q + 1] = rstd * (dv.y * gam[i][2 * q + 1] - a1 - (xv.y - mean) * rstd * a2);
        }
        if (has_r) {
          uint4 wr;
          asm volatile("ld.shared.v4.b32 {%0, %1, %2, %3}, [%4];" : "=r"(wr.x), "=r"(wr.y), "=r"(wr.z), "=r"(wr.w)
                       : "r"(slot(st, 2, i)));
          const uint32_t rs[4] = {wr.x, wr.y, wr.z, wr.w};
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            const float2 rv = unpack_bf16x2(rs[q]);
            o[2 * q] += rv.x;
            o[2 * q + 1] += rv.y;
            if constexpr (NACC == 4) {
              acc[2][i][2 * q] += rv.x;
              acc[2][i][2 * q + 1] += rv.y;
            }
          }
        }
        uint4 w;
        w.x = pack_bf16x2(o[0], o[1]);
        w.y = pack_bf16x2(o[2], o[3]);
        w.z = pack_bf16x2(o[4], o[5]);
        w.w = pack_bf16x2(o[6], o[7]);
        reinterpret_cast<uint4*>(dx + row * lddx)[j] = w;
        if constexpr (NACC == 4) {
          const uint32_t ws[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            const float2 ov = unpack_bf16x2(ws[q]);
            acc[3][i][2 * q] += ov.x;
            acc[3][i][2 * q + 1] += ov.y;
          }
        }
      }
    }
  }
  cp_async_wait_ln<0>();
  __syncthreads();  // every warp is done with its ring: reuse it for the reduction
  float* red = reinterpret_cast<float*>(smem_u8);  // [warp][NACC][C]
#pragma unroll
  for (int a = 0; a < NACC; ++a)
#pragma unroll
    for (int i = 0; i < V; ++i) {
      const int j = lane + 32 * i;
      if (j < nvec)
#pragma unroll
        for (int e = 0; e < 8; ++e) red[(warp * NACC + a) * C + j * 8 + e] = acc[a][i][e];
    }
  __syncthreads();
  for (int idx = threadIdx.x; idx < NACC * C; idx += kThreads) {
    float s = 0.f;
    for (int w = 0; w < kWarps; ++w) s += red[w * NACC * C + idx];
    partials[static_cast<long long>(blockIdx.x) * NACC * C + idx] = s;
  }
}

// out_a[c] (+)= sum_b partials[b][a][c] for each accumulator a with a non-null destination.
// Block = 32 columns x 8 row groups; each group sums a contiguous range of
// partial rows, then the 8 group sums are added in a fixed order.
// 32 columns per CTA, 32 warps: warp w sums a contiguous range of partial rows
// (loads unrolled, all in flight), then the 32 warp sums are added in order --
// a fixed summation order, so the result is the same on every rank.
__global__ void __launch_bounds__(1024) reduce_partials_kernel(const float* __restrict__ partials, int nblocks,
                                                              int nacc, int C, float* d0, float* d1, float* d2,
                                                              float* d3, int accumulate_mask) {
  pdl_trigger();  // the next kernel may launch now
  pdl_wait();     // global memory only after the previous kernel completed
  __shared__ float red[32][33];
  const int col = threadIdx.x & 31, grp = threadIdx.x >> 5;
  const int idx = blockIdx.x * 32 + col;
  const bool ok = idx < nacc * C;
  const int a = ok ? idx / C : 0, c = ok ? idx - a * C : 0;
  const int per = (nblocks + 31) / 32;
  const int b0 = grp * per, b1 = min(nblocks, b0 + per);
  float s = 0.f;
  if (ok) {
    const float* src = partials + static_cast<long long>(a) * C + c;
    const long long stride = static_cast<long long>(nacc) * C;
#pragma unroll 4
    for (int b = b0; b < b1; ++b) s += __ldg(src + b * stride);
  }
  red[grp][col] = s;
  __syncthreads();
  if (grp == 0 && ok) {
    float* dst = a == 0 ? d0 : a == 1 ? d1 : a == 2 ? d2 : d3;
    if (dst != nullptr) {
      float t = 0.f;
#pragma unroll
      for (int g = 0; g < 32; ++g) t += red[g][col];
      dst[c] = ((accumulate_mask >> a) & 1) ? dst[c] + t : t;
    }
  }
}

}  // namespace ln
}  // namespace md

namespace {
int g_sms = 0;
int sms() {
  if (g_sms == 0) {
    int dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&g_sms, cudaDevAttrMultiProcessorCount, dev);
  }
  return g_sms;
}

template <int T, int V>
cudaError_t ln_fwd_launch(const void* x, long long ldx, const float* g, const float* b, void* y, long long ldy,
                          float* mean, float* rstd, int M, int C, float eps, cudaStream_t s) {
  const int teams = md::ln::kThreads / T;
  int grid = (M + teams - 1) / teams;
  const int cap = sms() * 8;
  if (grid > cap) grid = cap;
  md::launch_pdl(md::ln::ln_fwd_kernel<T, V>, dim3(grid), dim3(md::ln::kThreads), 0, s,
      reinterpret_cast<const __nv_bfloat16*>(x), ldx, g, b, reinterpret_cast<__nv_bfloat16*>(y), ldy, mean, rstd, M,
      C, eps);
  return cudaGetLastError();
}

template <int T, int V, int NACC>
cudaError_t ln_bwd_launch(const void* dy, long long lddy, const void* x, long long ldx, const float* mean,
                          const float* rstd, const float* g, const void* rg, long long ldr, void* dx, long long lddx,
                          float* partials, int grid, int M, int C, cudaStream_t s) {
  const int teams = md::ln::kThreads / T;
  const size_t smem = (static_cast<size_t>(teams) * NACC * C + md::ln::kThreads / 32) * sizeof(float);
  auto kern = md::ln::ln_bwd_kernel<T, V, NACC>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
  if (e != cudaSuccess) return e;
  md::launch_pdl(kern, dim3(grid), dim3(md::ln::kThreads), smem, s,
      reinterpret_cast<const __nv_bfloat16*>(dy), lddy, reinterpret_cast<const __nv_bfloat16*>(x), ldx, mean, rstd, g,
      reinterpret_cast<const __nv_bfloat16*>(rg), ldr, reinterpret_cast<__nv_bfloat16*>(dx), lddx, partials, M, C);
  return cudaGetLastError();
}

template <int V>
cudaError_t ln_fwd_pipe_launch(const void* x, long long ldx, const float* g, const float* b, void* y, long long ldy,
                               float* mean, float* rstd, int M, int C, float eps, cudaStream_t s) {
  constexpr int kWarps = md::ln::kThreads / 32;
  const size_t smem = static_cast<size_t>(kWarps) * md::ln::kPipeStages * V * 32 * 16;
  auto kern = md::ln::ln_fwd_pipe_kernel<V>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
  if (e != cudaSuccess) return e;
  int grid = (M + kWarps - 1) / kWarps;
  const int cap = sms() * 2;  // 2 CTAs (16 warps) per SM: 48 rows in flight per SM
  if (grid > cap) grid = cap;
  md::launch_pdl(kern, dim3(grid), dim3(md::ln::kThreads), smem, s, reinterpret_cast<const __nv_bfloat16*>(x), ldx, g, b,
      reinterpret_cast<__nv_bfloat16*>(y), ldy, mean, rstd, M, C, eps);
  return cudaGetLastError();
}

template <int V, int NACC>
cudaError_t ln_bwd_pipe_launch(const void* dy, long long lddy, const void* x, long long ldx, const float* mean,
                               const float* rstd, const float* g, const void* rg, long long ldr, void* dx,
                               long long lddx, float* partials, int grid, int M, int C, cudaStream_t s) {
  constexpr int kWarps = md::ln::kThreads / 32;
  const size_t ring =
      static_cast<size_t>(kWarps) * md::ln::bwd_stages<V, NACC>() * (3 * V * 32 * 16 + 2 * sizeof(float));
  const size_t red = static_cast<size_t>(kWarps) * NACC * C * sizeof(float);
  const size_t smem = ring > red ? ring : red;
  auto kern = md::ln::ln_bwd_pipe_kernel<V, NACC>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
  if (e != cudaSuccess) return e;
  md::launch_pdl(kern, dim3(grid), dim3(md::ln::kThreads), smem, s,
      reinterpret_cast<const __nv_bfloat16*>(dy), lddy, reinterpret_cast<const __nv_bfloat16*>(x), ldx, mean, rstd, g,
      reinterpret_cast<const __nv_bfloat16*>(rg), ldr, reinterpret_cast<__nv_bfloat16*>(dx), lddx, partials, M, C);
  return cudaGetLastError();
}

bool ok16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }
}  // namespace

extern "C" {

// Number of CTAs (= partial rows) md_ln_bwd uses for M rows of width C.
int md_ln_bwd_grid(int M, int C, int nacc) {
  // The pipelined kernel holds two CTAs per SM up to C = 768 with two
  // accumulators (three-stage ring of 111 KB, 128 registers) and one
  // otherwise; the register kernel (C > 1024) runs two.
  int g = ((C <= 768 && nacc == 2) || C > 1024) ? sms() * 2 : sms();
  return g < M ? g : (M > 0 ? M : 1);
}

int md_ln_fwd(const void* x, long long ldx, const float* gamma, const float* beta, void* y, long long ldy, float* mean,
              float* rstd, int M, int C, float eps, cudaStream_t s) {
  if (M <= 0 || C <= 0 || (C % 8) || (ldx % 8) || (ldy % 8) || !ok16(x) || !ok16(y) || !ok16(gamma) || !ok16(beta))
    return -1;
  cudaError_t e;
  const int nvec = C / 8;
#define MD_LN_FWD_T(TT)                                                                  \
  {                                                                                      \
    const int v = (nvec + TT - 1) / TT;                                                  \
    if (v <= 1) e = ln_fwd_launch<TT, 1>(x, ldx, gamma, beta, y, ldy, mean, rstd, M, C, eps, s); \
    else if (v == 2) e = ln_fwd_launch<TT, 2>(x, ldx, gamma, beta, y, ldy, mean, rstd, M, C, eps, s); \
    else if (v == 3) e = ln_fwd_launch<TT, 3>(x, ldx, gamma, beta, y, ldy, mean, rstd, M, C, eps, s); \
    else e = ln_fwd_launch<TT, 4>(x, ldx, gamma, beta, y, ldy, mean, rstd, M, C, eps, s); \
  }
  if (C <= 1024) {
    const int v = (nvec + 31) / 32;
    if (v <= 1) e = ln_fwd_pipe_launch<1>(x, ldx, gamma, beta, y, ldy, mean, rstd, M, C, eps, s);
    else if (v == 2) e = ln_fwd_pipe_launch<2>(x, ldx, gamma, beta, y, ldy, mean, rstd, M, C, eps, s);
    else if (v == 3) e = ln_fwd_pipe_launch<3>(x, ldx, gamma, beta, y, ldy, mean, rstd, M, C, eps, s);
    else e = ln_fwd_pipe_launch<4>(x, ldx, gamma, beta, y, ldy, mean, rstd, M, C, eps, s);
  }
  else if (C <= 2048) MD_LN_FWD_T(64)
  else if (C <= 4096) MD_LN_FWD_T(128)
  else if (C <= 8192) MD_LN_FWD_T(256)
  else return -2;
#undef MD_LN_FWD_T
  return static_cast<int>(e);
}

// dx = LN'(dy) (+ resid_grad); partials [grid, nacc, C] (grid from md_ln_bwd_grid).
int md_ln_bwd(const void* dy, long long lddy, const void* x, long long ldx, const float* mean, const float* rstd,
              const float* gamma, const void* resid_grad, long long ldr, void* dx, long long lddx, float* partials,
              int nacc, int M, int C, cudaStream_t s) {
  if (M <= 0 || C <= 0 || (C % 8) || (lddy % 8) || (ldx % 8) || (lddx % 8) || !ok16(dy) || !ok16(x) || !ok16(dx) ||
      !ok16(gamma))
    return -1;
  if (resid_grad != nullptr && ((ldr % 8) || !ok16(resid_grad))) return -1;
  if (nacc != 2 && nacc != 4) return -3;
  if (nacc == 4 && resid_grad == nullptr) return -4;
  const int grid = md_ln_bwd_grid(M, C, nacc);
  cudaError_t e;
  const int nvec = C / 8;
#define MD_LN_BWD_TV(TT, VV)                                                                                      \
  (nacc == 2 ? ln_bwd_launch<TT, VV, 2>(dy, lddy, x, ldx, mean, rstd, gamma, resid_grad, ldr, dx, lddx, partials, \
                                        grid, M, C, s)                                                            \
             : ln_bwd_launch<TT, VV, 4>(dy, lddy, x, ldx, mean, rstd, gamma, resid_grad, ldr, dx, lddx, partials, \
                                        grid, M, C, s))
#define MD_LN_BWD_T(TT)                         \
  {                                             \
    const int v = (nvec + TT - 1) / TT;         \
    if (v <= 1) e = MD_LN_BWD_TV(TT, 1);        \
    else if (v == 2) e = MD_LN_BWD_TV(TT, 2);   \
    else if (v == 3) e = MD_LN_BWD_TV(TT, 3);   \
    else e = MD_LN_BWD_TV(TT, 4);               \
  }
#define MD_LN_BWD_PIPE(VV)                                                                                          \
  (nacc == 2 ? ln_bwd_pipe_launch<VV, 2>(dy, lddy, x, ldx, mean, rstd, gamma, resid_grad, ldr, dx, lddx, partials,   \
                                         grid, M, C, s)                                                              \
             : ln_bwd_pipe_launch<VV, 4>(dy, lddy, x, ldx, mean, rstd, gamma, resid_grad, ldr, dx, lddx, partials,   \
                                         grid, M, C, s))
  if (C <= 1024) {
    const int v = (nvec + 31) / 32;
    if (v <= 1) e = MD_LN_BWD_PIPE(1);
    else if (v == 2) e = MD_LN_BWD_PIPE(2);
    else if (v == 3) e = MD_LN_BWD_PIPE(3);
    else e = MD_LN_BWD_PIPE(4);
  }
  else if (C <= 2048) MD_LN_BWD_T(64)
  else if (C <= 4096) MD_LN_BWD_T(128)
  else if (C <= 8192) MD_LN_BWD_T(256)
  else return -2;
#undef MD_LN_BWD_T
#undef MD_LN_BWD_TV
#undef MD_LN_BWD_PIPE
  return static_cast<int>(e);
}

int md_ln_reduce(const float* partials, int nblocks, int nacc, int C, float* d0, float* d1, float* d2, float* d3,
                 int accumulate_mask, cudaStream_t s) {
  const int total = nacc * C;
  md::launch_pdl(md::ln::reduce_partials_kernel, dim3((total + 31) / 32), dim3(1024), 0, s, partials, nblocks, nacc, C, d0, d1, d2, d3,
      accumulate_mask);
  return static_cast<int>(cudaGetLastError());
}

}  // extern "C"
