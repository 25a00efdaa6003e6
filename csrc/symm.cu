// Symmetric peer memory and the peer-memory all-reduce kernel.
//
// Runtime: each rank allocates a buffer with cudaMalloc, exports a CUDA IPC
// handle, the handles are exchanged through torch.distributed, and every rank
// maps every peer's buffer (cudaIpcOpenMemHandle).  Kernels then read and write
// peer memory directly over NVLink / NVSwitch.  A second, small mapped buffer
// per rank holds barrier flags.
//
// md_ar_bucket_kernel — in-place all-reduce of `n` fp32 elements that sit at
// the same offset in every rank's buffer, scaled by `scale` (1/W for gradient
// averaging), in one launch:
//   1. arrive : CTA b of every rank raises its flag on every peer and waits for
//               the peers' CTA b (so all ranks' inputs are final);
//   2. reduce : rank r owns slice r of the range; CTA b sums its part of slice
//               r over all ranks in rank order 0..W-1 (bit-identical result on
//               every rank), scales it, and stores the result into slice r of
//               every rank's buffer (reduce-scatter and all-gather in one pass,
//               peer loads + peer stores);
//   3. depart : flags again, so no rank reads its buffer before every slice has
//               landed.
// Flags carry monotonically increasing epochs (2e+1 arrive, 2e+2 depart), so
// nothing is ever reset; the epoch is counted on the device per (flag page,
// channel), so kernels captured in a CUDA graph stay correct on replay.
//
// CTA pairing uses a *virtual* CTA index, taken from a per-channel counter in
// this rank's flag page in the order the CTAs become resident (the last CTA of
// a launch resets the counter).  Pairing by blockIdx.x would deadlock when
// another cross-rank kernel holds some SMs: rank A could have CTAs 0..k
// resident while rank B has CTAs k+1.. resident, each waiting for the other.
// With claimed indices the resident CTAs of every rank are always 0..k-1 for
// some k, so they pair up, finish and make room for the rest.  Every wait is bounded by a %globaltimer deadline; a
// wait that expires records kTimeoutPeer in the status word and the kernel
// returns.
//
// This is the fused replacement of the reference's per-bucket
// "copy grads, mul_(1/W), NCCL all_reduce, copy back" (ddp.py:75-101, 243-247).
#include "md_sm100.cuh"

namespace md {
namespace symm {

constexpr int kMaxWorld = 8;
constexpr int kMaxCtas = 160;     // flag slots per channel (one CTA per SM for the shard kernel)
constexpr int kArMaxCtas = 64;    // bucket all-reduce: leaves SMs to the backward it overlaps
constexpr int kChannels = 8;

// Peer-wait counters (analysis; off unless md_peer_wait_enable(1)): per
// channel, {CTA run ns, CTA ns spent in cross-rank barriers, launches}.
__device__ int g_pw_on;
__device__ unsigned long long g_pw[kChannels][3];

}  // namespace symm
}  // namespace md

struct MdArParams {
  float* bufs[md::symm::kMaxWorld];     // base of every rank's data buffer (index = rank in group)
  uint32_t* flags[md::symm::kMaxWorld];  // base of every rank's flag buffer
  long long offset;                      // element offset of the range in every buffer
  long long n;                           // elements (multiple of 4)
  int world, rank;
  float scale;
  int channel;                           // flag region (independent streams use different channels)
  unsigned long long timeout_ns;
  md::Status* status;
};

// Reduce-scatter of FSDP gradients (md_rs_shard): every rank holds the
// unit's full fp32 gradient at `offset` of its symmetric buffer; rank r sums
// elements [offset + r*shard, +shard) over all ranks (fixed rank order),
// scales by `scale`, and either writes / accumulates the result into its
// shard gradient `grad_out`, or (p != null) applies AdamW to its shard in
// place -- the reduce-scatter, 1/W scale, cast and optimizer update of the
// reference's fsdp.py:215-241 + optimizer.step() in one pass.
struct MdRsParams {
  float* bufs[md::symm::kMaxWorld];
  uint32_t* flags[md::symm::kMaxWorld];
  long long offset;      // element offset of the unit in every buffer
  long long shard;       // elements per rank (multiple of 4)
  int world, rank;
  float scale;
  int channel;
  unsigned long long timeout_ns;
  md::Status* status;
  float* grad_out;       // shard gradient, or null when p != null
  int accumulate;        // grad_out += result
  float* p;              // fused AdamW: fp32 shard, first moment, second moment
  float* m;
  float* v;
  float lr, b1, b2, eps, wd, bc1, bc2_sqrt;
  __nv_bfloat16* p_bf16; // fused AdamW: bf16 copy of the updated shard (the gather source), or null
};

// All-gather of FSDP parameter shards (md_ag_shards): every rank's fp32 shard
// of a unit sits at `offset` of its symmetric shard buffer; after an arrive
// barrier (every rank's shard is final) each rank copies all W shards into its
// own gathered buffer `out` (shard r at out[r * shard]), casting to bf16 when
// out_bf16 is set -- the reference's cast-then-all-gather (fsdp.py:172-182) as
// one pass of peer loads.  A depart barrier keeps any rank from updating its
// shard while a peer may still be reading it.
struct MdAgParams {
  const float* bufs[md::symm::kMaxWorld];
  uint32_t* flags[md::symm::kMaxWorld];
  long long offset;      // element offset of the unit's shard in every buffer
  long long shard;       // elements per rank (multiple of 4)
  int world, rank;
  int channel;
  unsigned long long timeout_ns;
  md::Status* status;
  void* out;             // world * shard elements, fp32 or bf16
  int out_bf16;
  int in_bf16;           // bufs hold bf16 shards (copied as they are; out must be bf16, shard % 8 == 0)
};

// Vocab-parallel cross-entropy statistics (md_ce_tp): each rank folds its
// [tiles, M] per-128-column (max, sum of exp) into per-row (max, sum) and
// publishes them with its target logit (0 where the target column belongs to
// another rank) at [0, M), [M, 2M), [2M, 3M) of its symmetric buffer; after
// the arrive barrier every rank combines all ranks' triples for its rows:
// lse = max + log(sum_r s_r exp(m_r - max)), loss = lse - sum_r t_r.  The
// reference's all_reduce(MAX) + two all_reduce(SUM) of [N]-sized tensors
// (tensor_parallel.py:457-474) as one kernel.
struct MdCeTpParams {
  float* bufs[md::symm::kMaxWorld];  // every rank's symmetric buffer, >= 3 * M floats
  uint32_t* flags[md::symm::kMaxWorld];
  int world, rank, channel;
  unsigned long long timeout_ns;
  md::Status* status;
  const float* tmax;  // this rank's [tiles, M] slab maxima
  const float* tsum;  // this rank's [tiles, M] slab sums of exp(x - max)
  int tiles;
  const float* ttgt;  // this rank's [M] target logits
  int M;
  float* lse;   // [M] out
  float* loss;  // [M] out (lse - target logit)
};

// Vocab-parallel embedding forward (md_embed_tp): every rank's bf16 shard of
// the token table sits in symmetric memory, so the token row for id lives on
// exactly one rank (the owner of its vocabulary range).  Each rank reads every
// row of its batch straight from the owner's shard over NVLink and adds the
// position row -- the reference's masked local lookup followed by an
// all-reduce of the [tokens, C] activations (tensor_parallel.py:409-416,
// gpt.py:183-185) as one gather that moves (W-1)/W of the rows once instead
// of 2(W-1)/W of them through a reduction.  An arrive barrier orders the
// reads after every owner's last shard update (its optimizer step is stream-
// ordered before this launch); a depart barrier keeps an owner from updating
// its shard while a peer may still be reading it.
struct MdEmbTpParams {
  const __nv_bfloat16* wte[md::symm::kMaxWorld];  // every rank's [vocab_rows, ldw] bf16 shard
  uint32_t* flags[md::symm::kMaxWorld];
  int world, rank, channel;
  unsigned long long timeout_ns;
  md::Status* status;
  const long long* ids;       // [M] token ids (global vocabulary)
  const __nv_bfloat16* wpe;   // [>= S, ldp] position rows (local)
  long long ldp;
  __nv_bfloat16* out;         // [M, ldo]
  long long ldo;
  long long ldw;
  long long vocab_rows;       // rows per shard (vocab / world)
  int M, S, C;                // C a multiple of 8
};

namespace md {
namespace symm {

__device__ __forceinline__ void st_release_sys(uint32_t* p, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// Flag index: [channel][cta][source rank]
__device__ __forceinline__ size_t flag_idx(int channel, int cta, int src) {
  return (static_cast<size_t>(channel) * kMaxCtas + cta) * kMaxWorld + src;
}

// {claimed, finished, launches} counters of `channel`, behind the flag slots
// of this rank's page.
template <typename P>
__device__ __forceinline__ uint32_t* vcta_counter(const P& p) {
  return p.flags[p.rank] + static_cast<size_t>(kChannels) * kMaxCtas * kMaxWorld + 3 * p.channel;
}

// Virtual index of this CTA (claim order; -1 if the counter is out of step)
// and the launch's epoch = launches on this (page, channel) so far + 1.  The
// epoch lives on the device so that a replayed CUDA graph advances it; every
// rank launches on a channel equally often, so the epochs agree across ranks.
struct VCta {
  int v;
  uint32_t epoch;
  uint64_t t0;  // %globaltimer at entry when the peer-wait counters are on, else 0
};
template <typename P>
__device__ VCta vcta_claim(const P& p) {
  __shared__ int v_sh;
  __shared__ uint32_t e_sh;
  __shared__ uint64_t t_sh;
  if (threadIdx.x == 0) {
    t_sh = g_pw_on ? globaltimer_ns() : 0ull;
    uint32_t* c = vcta_counter(p);
    const uint32_t v = atomicAdd(c, 1u);
    v_sh = v < gridDim.x ? static_cast<int>(v) : -1;
    if (v_sh < 0) report(p.status, kTimeoutPeer, 199, v);
    e_sh = *reinterpret_cast<volatile uint32_t*>(c + 2) + 1u;
  }
  __syncthreads();
  return VCta{v_sh, e_sh, t_sh};
}

// Every CTA calls this once on every exit path; the launch's last CTA records
// the epoch and resets the claim counters for the next launch on this channel
// (stream-ordered after it).
template <typename P>
__device__ void vcta_release(const P& p, const VCta& vct) {
  __syncthreads();
  if (threadIdx.x == 0) {
    const bool counting = vct.t0 != 0ull;
    if (counting) atomicAdd(&g_pw[p.channel][0], globaltimer_ns() - vct.t0);
    uint32_t* c = vcta_counter(p);
    if (atomicAdd(c + 1, 1u) == gridDim.x - 1) {
      atomicExch(c + 2, vct.epoch);
      atomicExch(c, 0u);
      atomicExch(c + 1, 0u);
      if (counting) atomicAdd(&g_pw[p.channel][2], 1ull);
    }
  }
}

// Per-CTA all-to-all barrier with the same virtual CTA `v` of every rank.
// Returns false on timeout (status recorded).
template <typename P>
__device__ bool cta_barrier(const P& p, int v, uint32_t value, uint32_t where) {
  __shared__ int ok_sh;
  __shared__ uint64_t tw_sh;
  if (threadIdx.x == 0) {
    ok_sh = 1;
    tw_sh = g_pw_on ? globaltimer_ns() : 0ull;
  }
  __syncthreads();
  const int peer = threadIdx.x;
  if (peer < p.world) {
    // The release store orders this CTA's earlier writes (ordered before it by
    // the __syncthreads above) at system scope; no separate fence needed.
    st_release_sys(p.flags[peer] + flag_idx(p.channel, v, p.rank), value);
    const uint32_t* mine = p.flags[p.rank] + flag_idx(p.channel, v, peer);
    const uint64_t t0 = globaltimer_ns();
    uint32_t it = 0;
    while (static_cast<int32_t>(ld_acquire_sys(mine) - value) < 0) {
      if ((++it & 255u) == 0 && globaltimer_ns() - t0 > p.timeout_ns) {
        report(p.status, kTimeoutPeer, where, static_cast<uint32_t>(peer));
        ok_sh = 0;
        break;
      }
    }
  }
  __syncthreads();
  if (threadIdx.x == 0 && tw_sh != 0ull) atomicAdd(&g_pw[p.channel][1], globaltimer_ns() - tw_sh);
  return ok_sh != 0;
}

__global__ void __launch_bounds__(512) md_ar_bucket_kernel(const __grid_constant__ MdArParams p) {
  const VCta vct = vcta_claim(p);
  const int vc = vct.v;
  const uint32_t arrive = 2u * vct.epoch + 1u, depart = 2u * vct.epoch + 2u;
  if (vc >= 0 && cta_barrier(p, vc, arrive, 100)) {

  const long long n4 = p.n / 4;
  const long long per = (n4 + p.world - 1) / p.world;
  const long long lo = static_cast<long long>(p.rank) * per;
  const long long hi = lo + per < n4 ? lo + per : n4;
  const long long stride = static_cast<long long>(gridDim.x) * blockDim.x;
  float4* bases[kMaxWorld];
#pragma unroll
  for (int r = 0; r < kMaxWorld; ++r)
    bases[r] = r < p.world ? reinterpret_cast<float4*>(p.bufs[r] + p.offset) : nullptr;

  // Two vectors per thread per step, every rank's loads of both issued before
  // any sum: twice the bytes in flight per thread (NVLink latency is ~us).
  for (long long u = lo + static_cast<long long>(vc) * blockDim.x + threadIdx.x; u < hi; u += 2 * stride) {
    const long long u2 = u + stride;
    const bool two = u2 < hi;
    float4 v[kMaxWorld], w[kMaxWorld];
#pragma unroll
    for (int r = 0; r < kMaxWorld; ++r)
      if (r < p.world) {
        v[r] = __ldcg(bases[r] + u);
        if (two) w[r] = __ldcg(bases[r] + u2);
      }
    float4 s = v[0], t = w[0];
#pragma unroll
    for (int r = 1; r < kMaxWorld; ++r)
      if (r < p.world) {
        s.x += v[r].x;
        s.y += v[r].y;
        s.z += v[r].z;
        s.w += v[r].w;
        t.x += w[r].x;
        t.y += w[r].y;
        t.z += w[r].z;
        t.w += w[r].w;
      }
    s.x *= p.scale;
    s.y *= p.scale;
    s.z *= p.scale;
    s.w *= p.scale;
    t.x *= p.scale;
    t.y *= p.scale;
    t.z *= p.scale;
    t.w *= p.scale;
#pragma unroll
    for (int r = 0; r < kMaxWorld; ++r)
      if (r < p.world) {
        __stcg(bases[r] + u, s);
        if (two) __stcg(bases[r] + u2, t);
      }
  }
  cta_barrier(p, vc, depart, 101);
  }
  vcta_release(p, vct);
}

__global__ void __launch_bounds__(512) md_rs_shard_kernel(const __grid_constant__ MdRsParams p) {
  const VCta vct = vcta_claim(p);
  const int vc = vct.v;
  const uint32_t arrive = 2u * vct.epoch + 1u, depart = 2u * vct.epoch + 2u;
  if (vc >= 0 && cta_barrier(p, vc, arrive, 110)) {
  const long long n4 = p.shard / 4;
  const long long base = (p.offset + static_cast<long long>(p.rank) * p.shard) / 4;
  const long long stride = static_cast<long long>(gridDim.x) * blockDim.x;
  const float4* srcs[kMaxWorld];
#pragma unroll
  for (int r = 0; r < kMaxWorld; ++r) srcs[r] = r < p.world ? reinterpret_cast<const float4*>(p.bufs[r]) + base : nullptr;
  const float step = p.lr / p.bc1, decay = 1.f - p.lr * p.wd;
  // Two vectors per thread per step (all loads of both issued first) to keep
  // enough bytes in flight for a streaming kernel.
  auto finish = [&](long long u, float4 s) {
    s.x *= p.scale;
    s.y *= p.scale;
    s.z *= p.scale;
    s.w *= p.scale;
    if (p.p != nullptr) {
      float4 pp = reinterpret_cast<float4*>(p.p)[u], mm = reinterpret_cast<float4*>(p.m)[u],
             vv = reinterpret_cast<float4*>(p.v)[u];
      float* P = &pp.x;
      float* M = &mm.x;
      float* V = &vv.x;
      const float* G = &s.x;
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        M[q] = p.b1 * M[q] + (1.f - p.b1) * G[q];
        V[q] = p.b2 * V[q] + (1.f - p.b2) * G[q] * G[q];
        P[q] = P[q] * decay - step * M[q] / (sqrtf(V[q]) / p.bc2_sqrt + p.eps);
      }
      reinterpret_cast<float4*>(p.p)[u] = pp;
      reinterpret_cast<float4*>(p.m)[u] = mm;
      reinterpret_cast<float4*>(p.v)[u] = vv;
      if (p.p_bf16 != nullptr)
        reinterpret_cast<uint2*>(p.p_bf16)[u] = make_uint2(pack_bf16x2(pp.x, pp.y), pack_bf16x2(pp.z, pp.w));
    } else {
      float4* g = reinterpret_cast<float4*>(p.grad_out) + u;
      if (p.accumulate) {
        const float4 o = *g;
        s.x += o.x;
        s.y += o.y;
        s.z += o.z;
        s.w += o.w;
      }
      *g = s;
    }
  };
  for (long long u = static_cast<long long>(vc) * blockDim.x + threadIdx.x; u < n4; u += 2 * stride) {
    const long long u2 = u + stride;
    const bool two = u2 < n4;
    float4 v[kMaxWorld], w[kMaxWorld];
#pragma unroll
    for (int r = 0; r < kMaxWorld; ++r)
      if (r < p.world) {
        v[r] = __ldcg(srcs[r] + u);
        if (two) w[r] = __ldcg(srcs[r] + u2);
      }
    float4 s = v[0], t = w[0];
#pragma unroll
    for (int r = 1; r < kMaxWorld; ++r)
      if (r < p.world) {
        s.x += v[r].x;
        s.y += v[r].y;
        s.z += v[r].z;
        s.w += v[r].w;
        t.x += w[r].x;
        t.y += w[r].y;
        t.z += w[r].z;
        t.w += w[r].w;
      }
    finish(u, s);
    if (two) finish(u2, t);
  }
  // No rank rewrites its gradient buffer before every peer has read it.
  cta_barrier(p, vc, depart, 111);
  }
  vcta_release(p, vct);
}

__global__ void __launch_bounds__(512) md_ag_shards_kernel(const __grid_constant__ MdAgParams p) {
  const VCta vct = vcta_claim(p);
  const int vc = vct.v;
  const uint32_t arrive = 2u * vct.epoch + 1u, depart = 2u * vct.epoch + 2u;
  if (vc >= 0 && cta_barrier(p, vc, arrive, 120)) {
  const long long n4 = p.shard / 4;
  const long long stride = static_cast<long long>(gridDim.x) * blockDim.x;
  // Rank by rank, starting at this rank's own shard so that at any time the W
  // ranks read from W different sources (no peer's links serve every reader);
  // four vectors per thread in flight (peer loads have ~us latency).
  constexpr int U = 4;
  if (p.in_bf16) {
    // bf16 shards (the optimizer keeps them next to the fp32 masters): 16-byte copies, no cast.
    const long long n8 = p.shard / 8;
    for (int step = 0; step < p.world; ++step) {
      const int r = (p.rank + step) % p.world;
      const uint4* src = reinterpret_cast<const uint4*>(reinterpret_cast<const __nv_bfloat16*>(p.bufs[r]) + p.offset);
      uint4* dst = reinterpret_cast<uint4*>(p.out) + static_cast<long long>(r) * n8;
      for (long long j = static_cast<long long>(vc) * blockDim.x + threadIdx.x; j < n8; j += U * stride) {
        uint4 a[U];
#pragma unroll
        for (int k = 0; k < U; ++k)
          if (j + k * stride < n8) a[k] = __ldcg(src + j + k * stride);
#pragma unroll
        for (int k = 0; k < U; ++k)
          if (j + k * stride < n8) dst[j + k * stride] = a[k];
      }
    }
  } else
  for (int step = 0; step < p.world; ++step) {
    const int r = (p.rank + step) % p.world;
    const float4* src = reinterpret_cast<const float4*>(p.bufs[r] + p.offset);
    const long long ob = static_cast<long long>(r) * n4;
    for (long long j = static_cast<long long>(vc) * blockDim.x + threadIdx.x; j < n4; j += U * stride) {
      float4 a[U];
#pragma unroll
      for (int k = 0; k < U; ++k)
        if (j + k * stride < n4) a[k] = __ldcg(src + j + k * stride);
#pragma unroll
      for (int k = 0; k < U; ++k) {
        const long long o = ob + j + k * stride;
        if (j + k * stride >= n4) break;
        if (p.out_bf16)
          reinterpret_cast<uint2*>(p.out)[o] = make_uint2(pack_bf16x2(a[k].x, a[k].y), pack_bf16x2(a[k].z, a[k].w));
        else
          reinterpret_cast<float4*>(p.out)[o] = a[k];
      }
    }
  }
  cta_barrier(p, vc, depart, 121);
  }
  vcta_release(p, vct);
}

__global__ void __launch_bounds__(256) md_ce_tp_kernel(const __grid_constant__ MdCeTpParams p) {
  constexpr float kLog2e = 1.4426950408889634f, kLn2 = 0.6931471805599453f;
  const VCta vct = vcta_claim(p);
  const int vc = vct.v;
  const uint32_t arrive = 2u * vct.epoch + 1u, depart = 2u * vct.epoch + 2u;
  if (vc >= 0) {
    const int per = (p.M + static_cast<int>(gridDim.x) - 1) / static_cast<int>(gridDim.x);
    const int lo = vc * per, hi = min(p.M, lo + per);
    float* mine = p.bufs[p.rank];
    for (int m = lo + threadIdx.x; m < hi; m += blockDim.x) {
      float mx = -INFINITY;
      for (int t = 0; t < p.tiles; ++t) mx = fmaxf(mx, p.tmax[static_cast<long long>(t) * p.M + m]);
      float s = 0.f;
      for (int t = 0; t < p.tiles; ++t) {
        const float tm = p.tmax[static_cast<long long>(t) * p.M + m];
        if (tm != -INFINITY) s += p.tsum[static_cast<long long>(t) * p.M + m] * exp2f((tm - mx) * kLog2e);
      }
      mine[m] = mx;
      mine[p.M + m] = s;
      mine[2 * p.M + m] = p.ttgt[m];
    }
    if (cta_barrier(p, vc, arrive, 130)) {
      for (int m = lo + threadIdx.x; m < hi; m += blockDim.x) {
        float mr[kMaxWorld], sr[kMaxWorld], tr = 0.f;
        float gmax = -INFINITY;
#pragma unroll
        for (int r = 0; r < kMaxWorld; ++r)
          if (r < p.world) {
            mr[r] = __ldcg(p.bufs[r] + m);
            sr[r] = __ldcg(p.bufs[r] + p.M + m);
            tr += __ldcg(p.bufs[r] + 2 * p.M + m);
            gmax = fmaxf(gmax, mr[r]);
          }
        float sum = 0.f;
#pragma unroll
        for (int r = 0; r < kMaxWorld; ++r)
          if (r < p.world && mr[r] != -INFINITY) sum += sr[r] * exp2f((mr[r] - gmax) * kLog2e);
        const float l = gmax + log2f(sum) * kLn2;
        p.lse[m] = l;
        p.loss[m] = l - tr;
      }
      // No rank rewrites its triples (next call) before every peer has read them.
      cta_barrier(p, vc, depart, 131);
    }
  }
  vcta_release(p, vct);
}

// One warp per token row, each lane moving 16 bytes per vector with up to 8
// peer loads in flight before any arithmetic (NVLink latency is ~1 us).
__global__ void __launch_bounds__(256) md_embed_tp_kernel(const __grid_constant__ MdEmbTpParams p) {
  const VCta vct = vcta_claim(p);
  const int vc = vct.v;
  const uint32_t arrive = 2u * vct.epoch + 1u, depart = 2u * vct.epoch + 2u;
  if (vc >= 0 && cta_barrier(p, vc, arrive, 140)) {
    const int warps = blockDim.x >> 5, warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int per = (p.M + static_cast<int>(gridDim.x) - 1) / static_cast<int>(gridDim.x);
    const int lo = vc * per, hi = min(p.M, lo + per);
    const int nvec = p.C / 8;
    constexpr int U = 8;
    for (int m = lo + warp; m < hi; m += warps) {
      const long long id = p.ids[m];
      long long owner = id / p.vocab_rows;
      if (owner >= p.world) owner = p.world - 1;
      const long long row = id - owner * p.vocab_rows;
      const bool valid = id >= 0 && row < p.vocab_rows;
      MD_CHECK(valid, p.status, 142, id);  // an id outside the vocabulary reads as a zero row
      const uint4* src = reinterpret_cast<const uint4*>(p.wte[valid ? owner : 0] + (valid ? row : 0) * p.ldw);
      const uint4* pos = reinterpret_cast<const uint4*>(p.wpe + static_cast<long long>(m % p.S) * p.ldp);
      uint4* dst = reinterpret_cast<uint4*>(p.out + static_cast<long long>(m) * p.ldo);
      for (int j0 = lane; j0 < nvec; j0 += 32 * U) {
        uint4 w[U];
#pragma unroll
        for (int k = 0; k < U; ++k) {
          const int j = j0 + 32 * k;
          w[k] = (valid && j < nvec) ? __ldcg(src + j) : make_uint4(0u, 0u, 0u, 0u);
        }
#pragma unroll
        for (int k = 0; k < U; ++k) {
          const int j = j0 + 32 * k;
          if (j >= nvec) break;
          const uint4 q = pos[j];
          const uint32_t a[4] = {w[k].x, w[k].y, w[k].z, w[k].w};
          const uint32_t b[4] = {q.x, q.y, q.z, q.w};
          uint32_t o[4];
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const float2 x = unpack_bf16x2(a[e]), y = unpack_bf16x2(b[e]);
            o[e] = pack_bf16x2(x.x + y.x, x.y + y.y);
          }
          dst[j] = make_uint4(o[0], o[1], o[2], o[3]);
        }
      }
    }
    cta_barrier(p, vc, depart, 141);
  }
  vcta_release(p, vct);
}

}  // namespace symm
}  // namespace md

extern "C" {

// Launch md_embed_tp_kernel with `ctas` CTAs (<= 160; the same count on every rank).
int md_embed_tp(const MdEmbTpParams* prm, int ctas, cudaStream_t s) {
  if (prm == nullptr || prm->world < 1 || prm->world > md::symm::kMaxWorld || prm->M <= 0 || prm->S <= 0 ||
      prm->C <= 0 || (prm->C % 8) || (prm->ldw % 8) || (prm->ldp % 8) || (prm->ldo % 8) || prm->vocab_rows <= 0 ||
      prm->out == nullptr || prm->ids == nullptr || prm->wpe == nullptr)
    return -1;
  if (ctas < 1 || ctas > md::symm::kMaxCtas || prm->channel < 0 || prm->channel >= md::symm::kChannels) return -2;
  md::symm::md_embed_tp_kernel<<<ctas, 256, 0, s>>>(*prm);
  return static_cast<int>(cudaGetLastError());
}

// Launch md_ce_tp_kernel with `ctas` CTAs (<= 160).
int md_ce_tp(const MdCeTpParams* prm, int ctas, cudaStream_t s) {
  if (prm == nullptr || prm->world < 1 || prm->world > md::symm::kMaxWorld || prm->M <= 0 || prm->tiles <= 0 ||
      prm->lse == nullptr || prm->loss == nullptr)
    return -1;
  if (ctas < 1 || ctas > md::symm::kMaxCtas || prm->channel < 0 || prm->channel >= md::symm::kChannels) return -2;
  md::symm::md_ce_tp_kernel<<<ctas, 256, 0, s>>>(*prm);
  return static_cast<int>(cudaGetLastError());
}

// Launch md_ag_shards_kernel with `ctas` CTAs (<= 160).
int md_ag_shards(const MdAgParams* prm, int ctas, cudaStream_t s) {
  if (prm == nullptr || prm->world < 1 || prm->world > md::symm::kMaxWorld || (prm->shard % 4) || (prm->offset % 4) ||
      prm->out == nullptr)
    return -1;
  if (prm->in_bf16 && (!prm->out_bf16 || (prm->shard % 8) || (prm->offset % 8))) return -1;
  if (ctas < 1 || ctas > md::symm::kMaxCtas || prm->channel < 0 || prm->channel >= md::symm::kChannels) return -2;
  md::symm::md_ag_shards_kernel<<<ctas, 512, 0, s>>>(*prm);
  return static_cast<int>(cudaGetLastError());
}

// Launch md_rs_shard_kernel with `ctas` CTAs (<= 64).
int md_rs_shard(const MdRsParams* prm, int ctas, cudaStream_t s) {
  if (prm == nullptr || prm->world < 1 || prm->world > md::symm::kMaxWorld || (prm->shard % 4) || (prm->offset % 4))
    return -1;
  if (ctas < 1 || ctas > md::symm::kMaxCtas || prm->channel < 0 || prm->channel >= md::symm::kChannels) return -2;
  if (prm->p == nullptr && prm->grad_out == nullptr) return -3;
  md::symm::md_rs_shard_kernel<<<ctas, 512, 0, s>>>(*prm);
  return static_cast<int>(cudaGetLastError());
}


// Peer-wait counters: on != 0 turns counting on (off otherwise) for the current
// device; reset != 0 zeroes the counters first.  Host-synchronous (analysis only).
int md_peer_wait_enable(int on, int reset) {
  if (reset) {
    unsigned long long zero[md::symm::kChannels][3] = {};
    cudaError_t e = cudaMemcpyToSymbol(md::symm::g_pw, zero, sizeof(zero));
    if (e != cudaSuccess) return static_cast<int>(e);
  }
  return static_cast<int>(cudaMemcpyToSymbol(md::symm::g_pw_on, &on, sizeof(int)));
}

// Copy the counters ([channel][run_ns, wait_ns, launches], 8 x 3) to host memory.
int md_peer_wait_read(unsigned long long* out) {
  return static_cast<int>(cudaMemcpyFromSymbol(out, md::symm::g_pw, sizeof(md::symm::g_pw)));
}

int md_symm_max_world() { return md::symm::kMaxWorld; }
long long md_symm_flag_bytes() {
  // Flag slots plus {claimed, finished, launches} counters per channel.
  return (static_cast<long long>(md::symm::kChannels) * md::symm::kMaxCtas * md::symm::kMaxWorld +
          3 * md::symm::kChannels) * sizeof(uint32_t);
}

// Allocate `bytes` of zeroed device memory and export its IPC handle (64 bytes into handle_out).
int md_symm_alloc(long long bytes, void** ptr_out, void* handle_out) {
  void* p = nullptr;
  cudaError_t e = cudaMalloc(&p, static_cast<size_t>(bytes));
  if (e != cudaSuccess) return static_cast<int>(e);
  e = cudaMemset(p, 0, static_cast<size_t>(bytes));
  if (e == cudaSuccess) e = cudaDeviceSynchronize();
  if (e == cudaSuccess) e = cudaIpcGetMemHandle(reinterpret_cast<cudaIpcMemHandle_t*>(handle_out), p);
  if (e != cudaSuccess) {
    cudaFree(p);
    return static_cast<int>(e);
  }
  *ptr_out = p;
  return 0;
}

int md_symm_open(const void* handle, void** ptr_out) {
  cudaIpcMemHandle_t h;
  memcpy(&h, handle, sizeof(h));
  return static_cast<int>(cudaIpcOpenMemHandle(ptr_out, h, cudaIpcMemLazyEnablePeerAccess));
}

int md_symm_close(void* peer_ptr) { return static_cast<int>(cudaIpcCloseMemHandle(peer_ptr)); }
int md_symm_free(void* ptr) { return static_cast<int>(cudaFree(ptr)); }

int md_allreduce_ctas(long long n, int world) {
  const long long per4 = (n / 4 + world - 1) / world;
  long long g = (per4 + 512 * 4 - 1) / (512 * 4);
  if (g < 1) g = 1;
  if (g > md::symm::kArMaxCtas) g = md::symm::kArMaxCtas;
  return static_cast<int>(g);
}

int md_allreduce(const MdArParams* prm, int ctas, cudaStream_t s) {
  if (prm == nullptr || prm->world < 1 || prm->world > md::symm::kMaxWorld || (prm->n % 4) || (prm->offset % 4))
    return -1;
  if (ctas < 1 || ctas > md::symm::kMaxCtas || prm->channel < 0 || prm->channel >= md::symm::kChannels) return -2;
  md::symm::md_ar_bucket_kernel<<<ctas, 512, 0, s>>>(*prm);
  return static_cast<int>(cudaGetLastError());
}

}  // extern "C"
