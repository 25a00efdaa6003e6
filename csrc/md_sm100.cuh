// Blackwell (sm_100a) device primitives shared by every kernel in this library:
// mbarriers with bounded waits, TMA tile loads (never multicast), tcgen05
// tensor-core MMA with TMEM accumulators, TMEM loads, and UMMA descriptors.
//
// Every wait in here is bounded by a %globaltimer deadline.  A wait that gives
// up records a status word (md::Status) and returns false; callers unwind
// instead of spinning forever, so a logic error shows up as an error code on
// the host rather than a hung GPU.
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <utility>

namespace md {

// ---------------------------------------------------------------------------
// Status word.  A kernel that gives up on a wait writes a code here; the host
// reads it with md_status_read().  Codes are small integers so several kernels
// can share one word with atomicMax (the first nonzero cause wins by value).
// ---------------------------------------------------------------------------
enum StatusCode : uint32_t {
  kOk = 0,
  kTimeoutPipeline = 1,   // intra-CTA producer/consumer mbarrier wait expired
  kTimeoutPeer = 2,       // cross-GPU flag wait expired
  kBadArgument = 3,       // kernel-side argument check failed
};

struct Status {
  uint32_t code;     // StatusCode
  uint32_t where;    // kernel-specific site id
  uint32_t block;    // blockIdx.x of the reporter
  uint32_t detail;   // e.g. expected epoch / peer rank
};

__device__ __forceinline__ void report(Status* st, uint32_t code, uint32_t where, uint32_t detail) {
  if (st == nullptr) return;
  if (atomicCAS(&st->code, 0u, code) == 0u) {
    st->where = where;
    st->block = blockIdx.x;
    st->detail = detail;
    __threadfence_system();
  }
}

// Index checks of the bounds-checking build (-DMD_BOUNDS_CHECK; nothing in the
// normal build): MD_CHECK(cond, where, detail) evaluates to `cond`, and when it
// is false records kBadArgument at site `where` with `detail` (the offending
// value, truncated) in the status word.  Callers skip the access on false; no
// kernel traps.
// Kernels without a status argument report into a per-file device word,
// g_md_check_status, read by that file's md_check_status_<file>() entry
// (MD_DEFINE_CHECK_READER).
#ifdef MD_BOUNDS_CHECK
#define MD_CHECK(cond, st, where, detail) \
  ((cond) ? true : (::md::report((st), ::md::kBadArgument, (where), static_cast<uint32_t>(detail)), false))
static __device__ ::md::Status g_md_check_status;
#define MD_CHECK_STATUS (&::md::g_md_check_status)
#define MD_DEFINE_CHECK_READER(name)                                                             \
  extern "C" int name(void* out, int reset) {                                                    \
    cudaError_t e = cudaMemcpyFromSymbol(out, ::md::g_md_check_status, sizeof(::md::Status));          \
    if (e == cudaSuccess && reset) {                                                             \
      ::md::Status z{};                                                                          \
      e = cudaMemcpyToSymbol(::md::g_md_check_status, &z, sizeof(z));                                  \
    }                                                                                            \
    return static_cast<int>(e);                                                                  \
  }
#else
#define MD_CHECK(cond, st, where, detail) true
#define MD_CHECK_STATUS nullptr
#define MD_DEFINE_CHECK_READER(name)                                                             \
  extern "C" int name(void* out, int reset) {                                                    \
    (void)reset;                                                                                 \
    memset(out, 0, sizeof(::md::Status));                                                        \
    return 0;                                                                                    \
  }
#endif

// Programmatic dependent launch.  A kernel launched with launch_pdl() may
// start while the previous kernel on its stream is still finishing: its CTAs
// run their prologue (barrier init, TMEM allocation) on SMs the predecessor
// has already left, then pdl_wait() blocks until the predecessor has completed
// and its memory is visible.  Every such kernel calls pdl_wait() before its
// first global-memory access; pdl_trigger() lets the NEXT kernel launch early.
// (Both are no-ops for a kernel launched without the attribute.)
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

// Whether launch_pdl() sets the attribute (environment MINIDIST_PDL=0 turns it off).
bool pdl_enabled();

template <typename... KArgs, typename... Args>
inline cudaError_t launch_pdl(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t stream,
                              Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl_enabled() ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, kern, std::forward<Args>(args)...);
}

__device__ __forceinline__ uint64_t globaltimer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// Intra-kernel pipeline waits never legitimately take more than milliseconds;
// two seconds means a protocol bug.
constexpr uint64_t kPipelineTimeoutNs = 2000000000ull;

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// ---------------------------------------------------------------------------
// mbarrier
// ---------------------------------------------------------------------------
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
               : "memory");
}

// Non-blocking probe: has the phase with this parity completed?  (mbar_try_wait
// may suspend the thread for a while; this never does, so a loop can poll
// several barriers.)
__device__ __forceinline__ bool mbar_test_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}\n"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}
__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}\n"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// Bounded wait on phase `parity`.  Returns false (and records a status) if the
// deadline passes.  `abort_flag` lets other roles in the CTA cut the wait short
// once one of them has already given up.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, Status* st, uint32_t where,
                                          volatile int* abort_flag) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = globaltimer_ns();
  for (uint32_t it = 0;; ++it) {
    if (mbar_try_wait(bar, parity)) return true;
    if ((it & 63u) == 63u) {
      if (abort_flag != nullptr && *abort_flag) return false;
      if (globaltimer_ns() - t0 > kPipelineTimeoutNs) {
        report(st, kTimeoutPipeline, where, parity);
        if (abort_flag != nullptr) *abort_flag = 1;
        return false;
      }
    }
  }
}

// ---------------------------------------------------------------------------
// TMA (cp.async.bulk.tensor) — plain tile loads into this CTA's shared memory.
// Every copy lands only in the issuing CTA's own shared memory.
// ---------------------------------------------------------------------------
__device__ __forceinline__ void tma_prefetch_desc(const CUtensorMap* map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

__device__ __forceinline__ void tma_load_2d(const CUtensorMap* map, uint64_t* bar, void* smem_dst, int c0,
                                            int c1) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4}], [%2];" ::"r"(smem_u32(smem_dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(c0), "r"(c1)
      : "memory");
}

// 3-D tile load; coordinates (c0 innermost).  Rows past a dimension's extent
// read as zero, which lets a [batch, seq, cols] view clip at each sequence end.
__device__ __forceinline__ void tma_load_3d(const CUtensorMap* map, uint64_t* bar, void* smem_dst, int c0, int c1,
                                            int c2) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4, %5}], [%2];" ::"r"(smem_u32(smem_dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(c0), "r"(c1), "r"(c2)
      : "memory");
}

__device__ __forceinline__ void tma_load_4d(const CUtensorMap* map, uint64_t* bar, void* smem_dst, int c0, int c1,
                                            int c2, int c3) {
  asm volatile(
      "cp.async.bulk.tensor.4d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4, %5, %6}], [%2];" ::"r"(smem_u32(smem_dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(c0), "r"(c1), "r"(c2), "r"(c3)
      : "memory");
}

// Bulk tensor reduce-add of a shared-memory tile into global memory (the
// tensor map's element type, e.g. fp32).  Elements outside the tensor's
// extent are skipped.  Completion is tracked with bulk groups.
__device__ __forceinline__ void tma_reduce_add_3d(const CUtensorMap* map, const void* smem_src, int c0, int c1,
                                                  int c2) {
  asm volatile(
      "cp.reduce.async.bulk.tensor.3d.global.shared::cta.add.tile.bulk_group [%0, {%2, %3, %4}], [%1];" ::"l"(
          reinterpret_cast<uint64_t>(map)),
      "r"(smem_u32(smem_src)), "r"(c0), "r"(c1), "r"(c2)
      : "memory");
}
__device__ __forceinline__ void tma_reduce_add_4d(const CUtensorMap* map, const void* smem_src, int c0, int c1,
                                                  int c2, int c3) {
  asm volatile(
      "cp.reduce.async.bulk.tensor.4d.global.shared::cta.add.tile.bulk_group [%0, {%2, %3, %4, %5}], [%1];" ::"l"(
          reinterpret_cast<uint64_t>(map)),
      "r"(smem_u32(smem_src)), "r"(c0), "r"(c1), "r"(c2), "r"(c3)
      : "memory");
}
// Bulk tensor store of a shared-memory tile to global memory (this GPU's own
// memory); elements outside the tensor's extent are not written.  The source
// must have been made visible to the async proxy (fence_proxy_async_smem by
// its writers, then a barrier).  Completion is tracked with bulk groups.
__device__ __forceinline__ void tma_store_3d(const CUtensorMap* map, const void* smem_src, int c0, int c1, int c2) {
  asm volatile("cp.async.bulk.tensor.3d.global.shared::cta.bulk_group [%0, {%2, %3, %4}], [%1];" ::"l"(
                   reinterpret_cast<uint64_t>(map)),
               "r"(smem_u32(smem_src)), "r"(c0), "r"(c1), "r"(c2)
               : "memory");
}
__device__ __forceinline__ void tma_store_4d(const CUtensorMap* map, const void* smem_src, int c0, int c1, int c2,
                                             int c3) {
  asm volatile("cp.async.bulk.tensor.4d.global.shared::cta.bulk_group [%0, {%2, %3, %4, %5}], [%1];" ::"l"(
                   reinterpret_cast<uint64_t>(map)),
               "r"(smem_u32(smem_src)), "r"(c0), "r"(c1), "r"(c2), "r"(c3)
               : "memory");
}
__device__ __forceinline__ void bulk_commit_group() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
// Wait until every committed bulk group has finished reading shared memory.
__device__ __forceinline__ void bulk_wait_read_all() { asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory"); }
// Wait until every committed bulk group has completed.
__device__ __forceinline__ void bulk_wait_all() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }

// Make this thread's generic-proxy shared-memory writes visible to the async
// proxy (tensor-core operand reads, TMA stores) that is ordered after it.
__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// ---------------------------------------------------------------------------
// tcgen05: TMEM allocation, MMA, commit, loads, fences
// ---------------------------------------------------------------------------
__device__ __forceinline__ void tmem_alloc(uint32_t* smem_result, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(smem_result)),
               "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tmem_relinquish() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}

__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// D[tmem] (+)= A[smem desc] * B[smem desc]^T, bf16 inputs, fp32 accumulate.
__device__ __forceinline__ void umma_bf16_ss(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                             uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}\n" ::"r"(tmem_d),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// Warp-uniform variants: every lane of a converged warp executes the call and
// elect.sync picks the issuing lane (always the lowest lane of a converged
// warp, so the same thread issues the MMAs and the commits that track them).
// Keeping the issuing loop warp-uniform lets the compiler hold descriptors and
// counters in uniform registers instead of converting them before every MMA.
__device__ __forceinline__ void umma_bf16_ss_elect(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                                   uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p, e;\n\t.reg .b32 r;\n\t"
      "elect.sync r|e, 0xffffffff;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "@e tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}\n" ::"r"(tmem_d),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}
// D (TMEM) (+)= A (TMEM) * B (shared memory), bf16 inputs, fp32 accumulate.  A
// occupies the 128 lanes from column tmem_a: row i of A in lane i, K-major,
// two bf16 per 32-bit column (8 columns per K = 16 step).  One elected lane issues.
__device__ __forceinline__ void umma_bf16_ts_elect(uint32_t tmem_d, uint32_t tmem_a, uint64_t bdesc, uint32_t idesc,
                                                   uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p, e;\n\t.reg .b32 r;\n\t"
      "elect.sync r|e, 0xffffffff;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "@e tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}\n" ::"r"(tmem_d),
      "r"(tmem_a), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}
__device__ __forceinline__ void umma_commit_elect(uint64_t* bar) {
  asm volatile(
      "{\n\t.reg .pred e;\n\t.reg .b32 r;\n\t"
      "elect.sync r|e, 0xffffffff;\n\t"
      "@e tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];\n\t}\n" ::"r"(smem_u32(bar))
      : "memory");
}

// Arrive on `bar` once every previously issued tcgen05.mma of this thread has
// completed (which also means their shared-memory operands may be reused).
__device__ __forceinline__ void umma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                   smem_u32(bar))
               : "memory");
}

__device__ __forceinline__ void tmem_ld_wait() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

// One warp reads 32 TMEM lanes x 32 consecutive 32-bit columns; thread i gets
// lane (base_lane + i), columns [col, col+32).
__device__ __forceinline__ void tmem_ld_32x32b_x32(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, "
      "%16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]),
        "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]),
        "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]),
        "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
}

// Inverse of tmem_ld_32x32b_x32: thread i writes lane (base_lane + i).
__device__ __forceinline__ void tmem_st_32x32b_x32(uint32_t taddr, const uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], "
      "{%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, %16, "
      "%17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31, %32};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]),
      "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15]), "r"(r[16]),
      "r"(r[17]), "r"(r[18]), "r"(r[19]), "r"(r[20]), "r"(r[21]), "r"(r[22]), "r"(r[23]), "r"(r[24]),
      "r"(r[25]), "r"(r[26]), "r"(r[27]), "r"(r[28]), "r"(r[29]), "r"(r[30]), "r"(r[31])
      : "memory");
}
__device__ __forceinline__ void tmem_st_32x32b_x16(uint32_t taddr, const uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], "
      "{%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, %16};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]),
      "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15])
      : "memory");
}
__device__ __forceinline__ void tmem_st_wait() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

// ---------------------------------------------------------------------------
// UMMA descriptors.
//
// Shared-memory matrix descriptor (64 bit): start address >> 4 in bits [0,14),
// leading-dimension byte offset >> 4 in [16,30), stride-dimension byte offset
// >> 4 in [32,46), descriptor version 1 in [46,48), base offset 0, layout type
// in [61,64) (2 = 128-byte swizzle).  With 128B swizzle:
//   K-major : rows of 128 B (64 bf16 along K), 8-row atoms 1024 B apart (SBO);
//             LBO unused.  Step along K inside the atom by adding bytes to the
//             start address.
//   MN-major: each K index is a 128 B row of 64 MN-elements; 8 K-rows make a
//             1024 B atom (SBO = 1024); consecutive 64-wide MN chunks are LBO
//             bytes apart.
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint64_t sdesc_sw128(uint32_t saddr, uint32_t lbo_bytes, uint32_t sbo_bytes) {
  uint64_t d = 0;
  d |= static_cast<uint64_t>((saddr & 0x3FFFFu) >> 4);
  d |= static_cast<uint64_t>((lbo_bytes >> 4) & 0x3FFFu) << 16;
  d |= static_cast<uint64_t>((sbo_bytes >> 4) & 0x3FFFu) << 32;
  d |= static_cast<uint64_t>(1) << 46;
  d |= static_cast<uint64_t>(2) << 61;
  return d;
}

// Instruction descriptor for kind::f16 with bf16 A/B and fp32 D.
// c_format bits [4,6)=1 (F32); a_format [7,10)=1 (BF16); b_format [10,13)=1;
// a_major bit 15, b_major bit 16 (1 = MN-major); N>>3 in [17,23); M>>4 in [24,29).
__host__ __device__ constexpr uint32_t idesc_bf16_f32(int M, int N, bool a_mn_major, bool b_mn_major) {
  return (1u << 4) | (1u << 7) | (1u << 10) | ((a_mn_major ? 1u : 0u) << 15) | ((b_mn_major ? 1u : 0u) << 16) |
         (static_cast<uint32_t>(N >> 3) << 17) | (static_cast<uint32_t>(M >> 4) << 24);
}

// ---------------------------------------------------------------------------
// Small helpers
// ---------------------------------------------------------------------------
__device__ __forceinline__ bool elect_one_sync() {
  uint32_t pred = 0;
  asm volatile(
      "{\n\t.reg .b32 rx;\n\t.reg .pred px;\n\t"
      "elect.sync rx|px, %1;\n\t"
      "selp.u32 %0, 1, 0, px;\n\t}\n"
      : "=r"(pred)
      : "r"(0xFFFFFFFFu));
  return pred != 0;
}

// Hardware tanh approximation (PTX tanh.approx.f32, ~2^-11 relative error):
// plenty for values that are rounded to bf16 right after.
__device__ __forceinline__ float tanh_fast(float x) {
  float y;
  asm("tanh.approx.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// GELU, tanh form (Hendrycks & Gimpel 2016): 0.5 x (1 + tanh(sqrt(2/pi) (x + 0.044715 x^3))).
// gelu_tanh(x) = 0.5 x (1 + tanh(u)), u = k0 (x + k1 x^3) = x (k0 + k0 k1 x^2),
// written as fused multiply-adds (six operations with the tanh).
__device__ __forceinline__ float gelu_tanh(float x) {
  const float k0 = 0.7978845608028654f;  // sqrt(2/pi)
  const float k0k1 = 0.7978845608028654f * 0.044715f;
  const float u = x * fmaf(x * x, k0k1, k0);
  const float h = 0.5f * x;
  return fmaf(h, tanh_fast(u), h);
}

// d/dx of gelu_tanh = 0.5 (1 + t) + 0.5 x (1 - t^2) k0 (1 + 3 k1 x^2), t = tanh(u).
__device__ __forceinline__ float gelu_tanh_grad(float x) {
  const float k0 = 0.7978845608028654f;
  const float k0k1 = 0.7978845608028654f * 0.044715f;
  const float x2 = x * x;
  const float t = tanh_fast(x * fmaf(x2, k0k1, k0));
  const float a = fmaf(0.5f, t, 0.5f);
  const float b = x * fmaf(x2, 1.5f * k0k1, 0.5f * k0);  // 0.5 x k0 (1 + 3 k1 x^2)
  return fmaf(b, fmaf(-t, t, 1.0f), a);
}

// Byte offset of (row, 16-byte chunk) inside a tile of 128-byte rows laid
// out with the TMA 128B swizzle (chunk index XOR row % 8; 8-row groups 1024 B
// apart).  The tile base must be 1024-byte aligned.
__device__ __forceinline__ uint32_t sw128_off(int row, int chunk) {
  return static_cast<uint32_t>((row >> 3) * 1024 + (row & 7) * 128 + ((chunk ^ (row & 7)) << 4));
}

__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi) {
  __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&v);
}

__device__ __forceinline__ float2 unpack_bf16x2(uint32_t v) {
  __nv_bfloat162 b = *reinterpret_cast<__nv_bfloat162*>(&v);
  return __bfloat1622float2(b);
}

}  // namespace md
