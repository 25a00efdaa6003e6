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
// nothing is ever reset.  Every wait is bounded by a %globaltimer deadline; a
// wait that expires records kTimeoutPeer in the status word and the kernel
// returns.
//
// This is the fused replacement of the reference's per-bucket
// "copy grads, mul_(1/W), NCCL all_reduce, copy back" (ddp.py:75-101, 243-247).
#include "md_sm100.cuh"

namespace md {
namespace symm {

constexpr int kMaxWorld = 8;
constexpr int kMaxCtas = 64;
constexpr int kChannels = 8;

}  // namespace symm
}  // namespace md

struct MdArParams {
  float* bufs[md::symm::kMaxWorld];     // base of every rank's data buffer (index = rank in group)
  uint32_t* flags[md::symm::kMaxWorld];  // base of every rank's flag buffer
  long long offset;                      // element offset of the range in every buffer
  long long n;                           // elements (multiple of 4)
  int world, rank;
  float scale;
  uint32_t epoch;
  int channel;                           // flag region (independent streams use different channels)
  unsigned long long timeout_ns;
  md::Status* status;
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

// Per-CTA all-to-all barrier with the same-index CTA of every rank.
// Returns false on timeout (status recorded).
__device__ bool cta_barrier(const MdArParams& p, uint32_t value, uint32_t where) {
  __shared__ int ok_sh;
  if (threadIdx.x == 0) ok_sh = 1;
  __syncthreads();
  const int peer = threadIdx.x;
  if (peer < p.world) {
    __threadfence_system();
    st_release_sys(p.flags[peer] + flag_idx(p.channel, blockIdx.x, p.rank), value);
    const uint32_t* mine = p.flags[p.rank] + flag_idx(p.channel, blockIdx.x, peer);
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
  return ok_sh != 0;
}

__global__ void __launch_bounds__(512) md_ar_bucket_kernel(const __grid_constant__ MdArParams p) {
  const uint32_t arrive = 2u * p.epoch + 1u, depart = 2u * p.epoch + 2u;
  if (!cta_barrier(p, arrive, 100)) return;

  const long long n4 = p.n / 4;
  const long long per = (n4 + p.world - 1) / p.world;
  const long long lo = static_cast<long long>(p.rank) * per;
  const long long hi = lo + per < n4 ? lo + per : n4;
  const long long stride = static_cast<long long>(gridDim.x) * blockDim.x;
  float4* bases[kMaxWorld];
#pragma unroll
  for (int r = 0; r < kMaxWorld; ++r)
    bases[r] = r < p.world ? reinterpret_cast<float4*>(p.bufs[r] + p.offset) : nullptr;

  for (long long u = lo + static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x; u < hi; u += stride) {
    float4 v[kMaxWorld];
#pragma unroll
    for (int r = 0; r < kMaxWorld; ++r)
      if (r < p.world) v[r] = __ldcg(bases[r] + u);
    float4 s = v[0];
#pragma unroll
    for (int r = 1; r < kMaxWorld; ++r)
      if (r < p.world) {
        s.x += v[r].x;
        s.y += v[r].y;
        s.z += v[r].z;
        s.w += v[r].w;
      }
    s.x *= p.scale;
    s.y *= p.scale;
    s.z *= p.scale;
    s.w *= p.scale;
#pragma unroll
    for (int r = 0; r < kMaxWorld; ++r)
      if (r < p.world) __stcg(bases[r] + u, s);
  }
  cta_barrier(p, depart, 101);
}

}  // namespace symm
}  // namespace md

extern "C" {

int md_symm_max_world() { return md::symm::kMaxWorld; }
long long md_symm_flag_bytes() {
  return static_cast<long long>(md::symm::kChannels) * md::symm::kMaxCtas * md::symm::kMaxWorld * sizeof(uint32_t);
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
  if (g > 32) g = 32;
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
