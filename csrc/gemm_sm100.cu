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
// Two tile configurations share one kernel template:
//   CG = 1: one CTA per SM computes 128 x 256 output tiles (tcgen05 cta_group::1).
//   CG = 2: a cluster of two CTAs on two SMs computes 256 x 256 tiles with
//           cta_group::2 MMAs: each CTA stages its own 128 rows of A and half
//           (128 columns) of B, so per-SM operand traffic drops by a third;
//           the leader CTA issues the MMAs, each CTA's TMEM holds its 128 rows
//           of the accumulator.  Both CTAs' loads complete on the leader's
//           mbarrier; the leader's MMA completion is signalled to both CTAs'
//           barriers with one masked tcgen05.commit.
//
// Warp roles (64 + 32*EW threads):
//   warp 0       : TMA producer (one thread), 6-stage ring (CG=2) / 4 (CG=1)
//   warp 1       : TMEM allocator + MMA issuer (one thread, leader CTA only)
//   warps 2..    : EW epilogue warps; warp w reads TMEM lanes 32*(w%4)..+31;
//                  with EW = 8 two warps share a lane quarter and split the
//                  256 accumulator columns.
// 512 TMEM columns hold two 256-column fp32 accumulators, so the epilogue of
// tile i overlaps the main loop of tile i+1.
//
// Epilogues (EpiMode):
//   kEpiBF16  : (+bias) (-> store pre-activation, GELU) (+residual) -> bf16
//   kEpiF32   : fp32 store, optionally D += acc (gradient accumulation); with
//               k_splits > 1 each split writes a partial slab of `workspace`
//               and a fixed-order reduce kernel sums them
//   kEpiDGELU : acc * gelu'(pre-activation) -> bf16   (MLP backward)
//   kEpiCE    : bf16 logits plus per-(row, 128-column slab) max / sum-exp and
//               the target logit, for the fused cross-entropy
//
// Every mbarrier wait is bounded (md_sm100.cuh); on expiry the kernel records a
// status word, drains its own copies and MMAs, frees TMEM and returns.
//
// Replaces the reference's F.linear calls (tensor_parallel.py:291,354 via
// models/gpt.py) and, through kEpiCE, the logits half of
// _VocabParallelCrossEntropy (tensor_parallel.py:451-479).
#include <cudaTypedefs.h>

#include <cstdlib>

#include "md_sm100.cuh"

namespace md {
namespace gemm {

constexpr int BM = 128;  // rows per CTA
constexpr int BN = 256;  // columns per tile
constexpr int BK = 64;
constexpr int kABytes = BM * BK * 2;  // 16 KB
constexpr int kTmemCols = 512;
constexpr int kCeSlab = 128;  // CE statistics are kept per 128-column slab

enum EpiMode : int { kEpiBF16 = 0, kEpiF32 = 1, kEpiDGELU = 2, kEpiCE = 3 };

// Epilogue staging: each epilogue warp owns two slabs of 32 rows x 128 bytes
// (128B-swizzled) that TMA stores / reduce-adds write out (double-buffered
// output, or output + GELU pre-activation).  Eight epilogue warps (the
// heavy GELU / dGELU / cross-entropy epilogues) take 64 KB of staging, paid
// for with one mainloop stage less.
constexpr int kSlabBytes = 32 * 128;

template <int CG, int EW>
struct Cfg {
  static constexpr int kBBytes = (BN / CG) * BK * 2;  // B rows staged by this CTA
  static constexpr int kStageBytes = kABytes + kBBytes;
  static constexpr int kStages = EW == 8 ? (CG == 2 ? 5 : 3) : (CG == 2 ? 6 : 4);
  static constexpr int kEpiSmem = EW * 2 * kSlabBytes;
  static constexpr int kSmemBytes = 1024 + kStages * kStageBytes + kEpiSmem + 256;
  static_assert(kSmemBytes <= 232448, "shared memory budget");
};

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
  float* ce_max;               // [ceil(N/128), M]
  float* ce_sum;               // [ceil(N/128), M]
  float* ce_tgt;               // [M]
  long long ce_col_offset;     // global column id of this shard's column 0
  int num_sms;                 // grid cap (0 -> all SMs)
  md::Status* status;
  int cta_group;               // 0 = choose, 1 or 2
  int epi_warps;               // 0 = choose, 4 or 8
  // kEpiDGELU: per-32-row column sums of the (bf16-rounded) output, fp32
  // [ceil(M/32), N] -- the bias gradient's first stage, so the output is not
  // read back for it -- or null.
  float* colsum;
  // kEpiBF16 without bias / GELU / residual: row-wise dot products of the
  // (bf16-rounded) output with `dot_in` over groups of `dot_group` columns
  // (32, 64 or 128), written to dot_out[((row / dot_seq) * (N / dot_group) + g)
  // * dot_seq + row % dot_seq] -- the attention backward's
  // delta = rowsum(dO * O) per (batch, head, query) from the GEMM producing dO.
  const void* dot_in;          // bf16 [M, lddot] or null
  long long lddot;
  float* dot_out;
  int dot_group;
  int dot_seq;
};

// Fused tensor-parallel all-reduce of the GEMM output (md_gemm_ar): the
// epilogue writes this rank's partial tile (bf16) into its symmetric partial
// buffer and publishes a per-chunk ready flag; comm warps reduce the chunks
// this rank owns across all ranks (peer loads), add bias and residual once,
// write the result to the local output and to this rank's symmetric final
// buffer, publish a final flag, and copy every other chunk from its owner's
// final buffer.  A chunk is 32 rows x one 256-column tile; owner = id % world.
struct MdTpArParams {
  void* partial[8];      // every rank's partial buffer (bf16, row stride ldp)
  void* fin[8];          // every rank's final buffer (bf16, row stride ldp)
  unsigned* flags[8];    // every rank's flag page: ready[max_chunks], final[max_chunks]
  long long ldp;
  void* out;             // this rank's output (bf16, row stride ldo)
  long long ldo;
  const float* bias;     // [N] or null, added after the reduction
  const void* resid;     // bf16 [M, ldr] or null, added after the reduction
  long long ldr;
  int world, rank;
  unsigned epoch;        // flags carry epochs; a call waits for >= epoch
  int max_chunks;
  unsigned long long timeout_ns;
  unsigned long long* trace;  // optional analysis trace ([64][8] %globaltimer stamps of CTA 0), or null
  // This rank's {claimed, finished, epoch} counters (3 x u32; the first two are
  // zero between launches), or null for blockIdx order and the host's `epoch`.
  // With counters the epoch is the launch count + 1, read on the device, so a
  // replayed CUDA graph advances it.  Clusters take their tile-walk
  // index in the order they become resident, so when another kernel holds
  // some SMs the resident clusters of every rank are the same prefix 0..k-1
  // and pair up across ranks instead of waiting on clusters not yet running.
  unsigned* claim;
};

namespace md {

bool pdl_enabled() {
  static const int on = [] {
    const char* e = getenv("MINIDIST_PDL");
    return (e == nullptr || (e[0] != '0' && e[0] != 'n' && e[0] != 'f')) ? 1 : 0;
  }();
  return on != 0;
}

namespace gemm {

struct KParams {
  MdGemmParams p;
  int tiles_m;  // in units of CG*128 rows
  int tiles_n, units, k_blocks, kb_per_split;
  MdTpArParams ar;
};

__device__ __forceinline__ void decode_unit(const KParams& kp, int u, int& tm, int& tn, int& split) {
  const int per_split = kp.tiles_m * kp.tiles_n;
  split = u / per_split;
  const int rem = u - split * per_split;
  tm = rem / kp.tiles_n;
  tn = rem - tm * kp.tiles_n;
}

// ---------------------------------------------------------------------------
// Cluster helpers (CG = 2)
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint32_t cluster_ctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
__device__ __forceinline__ uint32_t map_to_cta(uint32_t smem_addr, uint32_t cta) {
  uint32_t out;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(out) : "r"(smem_addr), "r"(cta));
  return out;
}
__device__ __forceinline__ void mbar_arrive_remote(uint32_t cluster_addr) {
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(cluster_addr) : "memory");
}
__device__ __forceinline__ void cluster_sync() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
// TMA tile load into this CTA's shared memory whose transaction bytes are
// counted on the pair leader's mbarrier (cluster address).
__device__ __forceinline__ void tma_load_2d_pair(const CUtensorMap* map, uint32_t leader_bar, void* smem_dst, int c0,
                                                 int c1) {
  asm volatile(
      "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4}], [%2];" ::"r"(smem_u32(smem_dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(leader_bar), "r"(c0), "r"(c1)
      : "memory");
}
__device__ __forceinline__ void tmem_alloc_pair(uint32_t* smem_result, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(smem_result)),
               "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tmem_relinquish_pair() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc_pair(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
__device__ __forceinline__ void umma_bf16_ss_pair(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                                  uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n\t}\n" ::"r"(tmem_d),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}
// Arrive on the mbarrier at this shared-memory offset in both CTAs of the pair
// once the issuing thread's MMAs complete (commit with a CTA mask; this is a
// completion signal, not a data copy).
__device__ __forceinline__ void umma_commit_pair_both(uint64_t* bar) {
  const uint16_t mask = 0x3;
  asm volatile(
      "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%0], %1;" ::"r"(
          smem_u32(bar)),
      "h"(mask)
      : "memory");
}
__device__ __forceinline__ void umma_commit_pair(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}

// Warp-uniform issue: every lane of the MMA warp runs the loop, elect.sync
// picks the issuing lane (the same lowest lane every time, so it also owns the
// commits that track its MMAs), and descriptors stay in uniform registers.
template <int CG>
__device__ __forceinline__ void umma_elect(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                           uint32_t accumulate) {
  if constexpr (CG == 2) {
    asm volatile(
        "{\n\t.reg .pred p, e;\n\t.reg .b32 r;\n\t"
        "elect.sync r|e, 0xffffffff;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "@e tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n\t}\n" ::"r"(tmem_d),
        "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
        : "memory");
  } else {
    umma_bf16_ss_elect(tmem_d, adesc, bdesc, idesc, accumulate);
  }
}
// Commit that arrives on `bar` in every CTA of the pair (CG = 2) or this CTA.
template <int CG>
__device__ __forceinline__ void commit_all_elect(uint64_t* bar) {
  if constexpr (CG == 2) {
    const uint16_t mask = 0x3;
    asm volatile(
        "{\n\t.reg .pred e;\n\t.reg .b32 r;\n\t"
        "elect.sync r|e, 0xffffffff;\n\t"
        "@e tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%0], %1;\n\t}\n" ::"r"(
            smem_u32(bar)),
        "h"(mask)
        : "memory");
  } else {
    umma_commit_elect(bar);
  }
}
// Commit that arrives on `bar` in this (leader) CTA only.
template <int CG>
__device__ __forceinline__ void commit_self_elect(uint64_t* bar) {
  if constexpr (CG == 2) {
    asm volatile(
        "{\n\t.reg .pred e;\n\t.reg .b32 r;\n\t"
        "elect.sync r|e, 0xffffffff;\n\t"
        "@e tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.b64 [%0];\n\t}\n" ::"r"(smem_u32(bar))
        : "memory");
  } else {
    umma_commit_elect(bar);
  }
}

__device__ __forceinline__ float ex2_approx(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// ---------------------------------------------------------------------------
// Epilogue.  One thread owns one accumulator row (TMEM lane) and walks the
// 32-column chunks [c_begin, c_end) of the 256-column tile; the warp stages
// its 32 rows chunk by chunk in shared memory (128-byte rows, 128B swizzle,
// conflict-free) and one lane writes each full slab with a TMA store (bf16:
// 64 columns; fp32: 32 columns) or, when accumulating into D (beta, atomic
// split-K), a TMA reduce-add.  Rows past M and columns past N are clipped by
// the tensor map.  Every lane runs every step (tcgen05.ld, the staging and
// the __syncwarp are warp-collective).
// ---------------------------------------------------------------------------
struct EpiStage {
  uint8_t* base;  // this warp's slabs
  int nbuf;       // 1 or 2
  int ctr;        // slabs issued so far
  int lane;
};

__device__ __forceinline__ uint8_t* slab_acquire(EpiStage& e) {
  if (e.ctr >= e.nbuf) {
    if (e.lane == 0) {
      if (e.nbuf == 2) asm volatile("cp.async.bulk.wait_group.read 1;" ::: "memory");
      else asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory");
    }
    __syncwarp();
  }
  return e.base + (e.ctr % e.nbuf) * kSlabBytes;
}

// mode 0: store, 1: reduce-add; dims 2 (x, y) or 3 (x, y, z).
__device__ __forceinline__ void slab_issue(EpiStage& e, const CUtensorMap* map, const uint8_t* sb, int mode, int dims,
                                           int x, int y, int z) {
  fence_proxy_async_smem();
  __syncwarp();
  if (e.lane == 0) {
    const uint64_t m = reinterpret_cast<uint64_t>(map);
    const uint32_t a = smem_u32(sb);
    if (dims == 3) {
      if (mode == 1)
        asm volatile("cp.reduce.async.bulk.tensor.3d.global.shared::cta.add.tile.bulk_group [%0, {%2, %3, %4}], [%1];"
                     ::"l"(m), "r"(a), "r"(x), "r"(y), "r"(z) : "memory");
      else
        asm volatile("cp.async.bulk.tensor.3d.global.shared::cta.bulk_group [%0, {%2, %3, %4}], [%1];"
                     ::"l"(m), "r"(a), "r"(x), "r"(y), "r"(z) : "memory");
    } else {
      if (mode == 1)
        asm volatile("cp.reduce.async.bulk.tensor.2d.global.shared::cta.add.tile.bulk_group [%0, {%2, %3}], [%1];"
                     ::"l"(m), "r"(a), "r"(x), "r"(y) : "memory");
      else
        asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%2, %3}], [%1];"
                     ::"l"(m), "r"(a), "r"(x), "r"(y) : "memory");
    }
    bulk_commit_group();
  }
  ++e.ctr;
}

template <int EPI>
__device__ __forceinline__ void epilogue_row(const MdGemmParams& p, const CUtensorMap* tmD, const CUtensorMap* tmX,
                                             EpiStage& es, int row, int row0, int tn, int split, uint32_t t_row,
                                             int c_begin, int c_end) {
  const bool row_ok = row < p.M;
  const int lane = es.lane;
  long long tgt = -1;
  if (EPI == kEpiCE && row_ok) tgt = p.ce_target[row] - p.ce_col_offset;
  constexpr bool kF32 = EPI == kEpiF32;
  const bool to_ws = kF32 && p.k_splits > 1 && p.workspace != nullptr;
  const int f32_mode = (kF32 && !to_ws && (p.k_splits > 1 || p.beta)) ? 1 : 0;
  uint8_t* sb = nullptr;
  // Second input of the epilogue (the residual for kEpiBF16, the
  // pre-activation for kEpiDGELU), read one chunk ahead so its load latency
  // overlaps the current chunk instead of stalling every chunk.
  const __nv_bfloat16* in_base = nullptr;
  long long in_ld = 0;
  if (EPI == kEpiBF16 && p.resid != nullptr) {
    in_base = reinterpret_cast<const __nv_bfloat16*>(p.resid);
    in_ld = p.ldres;
  } else if (EPI == kEpiBF16 && p.dot_out != nullptr) {
    in_base = reinterpret_cast<const __nv_bfloat16*>(p.dot_in);
    in_ld = p.lddot;
  } else if (EPI == kEpiDGELU) {
    in_base = reinterpret_cast<const __nv_bfloat16*>(p.aux);
    in_ld = p.ldaux;
  }
  uint4 nxt[4];
  auto load_in = [&](int c) {
    const int n0 = tn * BN + c * 32;
    if (in_base != nullptr && row_ok && c < c_end && n0 + 32 <= p.N) {
      const uint4* src = reinterpret_cast<const uint4*>(in_base + row * in_ld + n0);
#pragma unroll
      for (int q = 0; q < 4; ++q) nxt[q] = src[q];
    }
  };
  load_in(c_begin);
  // The chunk's bias is loaded before its TMEM load, so the two latencies
  // overlap (a load at the point of use stalled every chunk on it).
  const bool bias_vec = EPI == kEpiBF16 && p.bias != nullptr && (reinterpret_cast<uintptr_t>(p.bias) & 15u) == 0;
  float dot_acc = 0.f;
#pragma unroll 1
  for (int slab = c_begin / 4; slab < c_end / 4; ++slab) {
    float ce_m = -INFINITY, ce_s = 0.f;
    bool ce_any = false;
#pragma unroll 1
    for (int c = slab * 4; c < slab * 4 + 4; ++c) {
      const int n0 = tn * BN + c * 32;
      if (n0 >= p.N) break;  // warp-uniform: the rest of this tile lies past N
      uint4 cur[4];
#pragma unroll
      for (int q = 0; q < 4; ++q) cur[q] = nxt[q];
      load_in(c + 1);
      float4 bcur[8];
      if (bias_vec) {
        if (n0 + 32 <= p.N) {
          const float4* b4 = reinterpret_cast<const float4*>(p.bias + n0);
#pragma unroll
          for (int q = 0; q < 8; ++q) bcur[q] = __ldg(b4 + q);
        } else {
          float* bf = reinterpret_cast<float*>(bcur);
#pragma unroll
          for (int j = 0; j < 32; ++j) bf[j] = n0 + j < p.N ? __ldg(p.bias + n0 + j) : 0.f;
        }
      }
      uint32_t r[32];
      tmem_ld_32x32b_x32(t_row + c * 32, r);
      tmem_ld_wait();
      const bool full = (n0 + 32 <= p.N);
      uint32_t ce_pk[EPI == kEpiCE ? 16 : 1];
      float v[32];
      if (p.alpha != 1.f) {  // warp-uniform
#pragma unroll
        for (int j = 0; j < 32; ++j) v[j] = __uint_as_float(r[j]) * p.alpha;
      } else {
#pragma unroll
        for (int j = 0; j < 32; ++j) v[j] = __uint_as_float(r[j]);
      }

      if (EPI == kEpiBF16) {
        if (bias_vec) {
          const float* bf = reinterpret_cast<const float*>(bcur);
#pragma unroll
          for (int j = 0; j < 32; ++j) v[j] += bf[j];
        } else if (p.bias != nullptr) {
#pragma unroll
          for (int j = 0; j < 32; ++j) v[j] += (n0 + j < p.N) ? p.bias[n0 + j] : 0.f;
        }
        if (p.gelu) {
          // The pre-activation, rounded to bf16 once: packed pairs are stored
          // and unpacked back, so backward differentiates exactly this value.
          uint32_t pk[16];
#pragma unroll
          for (int q = 0; q < 16; ++q) pk[q] = pack_bf16x2(v[2 * q], v[2 * q + 1]);
#pragma unroll
          for (int q = 0; q < 16; ++q) {
            v[2 * q] = __uint_as_float(pk[q] << 16);
            v[2 * q + 1] = __uint_as_float(pk[q] & 0xFFFF0000u);
          }
          // The pre-activation goes out through the second slab of this warp
          // (TMA store on tmX at the end of the slab); see the staging below.
          if ((c & 1) == 0) {
            if (es.ctr > 0) {
              if (lane == 0) asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory");
              __syncwarp();
            }
            sb = es.base;
          }
#pragma unroll
          for (int q = 0; q < 4; ++q)
            asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(
                             smem_u32(es.base + kSlabBytes + sw128_off(lane, (c & 1) * 4 + q))),
                         "r"(pk[4 * q]), "r"(pk[4 * q + 1]), "r"(pk[4 * q + 2]), "r"(pk[4 * q + 3])
                         : "memory");
          // GELU of the bf16-rounded pre-activation: exactly what backward differentiates.
#pragma unroll
          for (int j = 0; j < 32; ++j) v[j] = gelu_tanh(v[j]);
        }
        if (p.dot_out != nullptr) {
          // Dot product of this row's bf16 output with dot_in over the group.
          if (row_ok && full) {
#pragma unroll
            for (int q = 0; q < 4; ++q) {
              const uint4 w = cur[q];
              const float2 f0 = unpack_bf16x2(w.x), f1 = unpack_bf16x2(w.y), f2 = unpack_bf16x2(w.z),
                           f3 = unpack_bf16x2(w.w);
              const float o[8] = {f0.x, f0.y, f1.x, f1.y, f2.x, f2.y, f3.x, f3.y};
#pragma unroll
              for (int e = 0; e < 8; ++e) dot_acc += __bfloat162float(__float2bfloat16_rn(v[q * 8 + e])) * o[e];
            }
          }
          const int gsz = p.dot_group >> 5;  // chunks per group
          if ((c + 1) % gsz == 0) {
            if (row_ok) {
              const int g = (n0 + 32) / p.dot_group - 1;
              const long long b = row / p.dot_seq, q = row % p.dot_seq;
              p.dot_out[(b * (p.N / p.dot_group) + g) * p.dot_seq + q] = dot_acc;
            }
            dot_acc = 0.f;
          }
        }
        if (p.resid != nullptr && row_ok) {
          const __nv_bfloat16* rs = reinterpret_cast<const __nv_bfloat16*>(p.resid) + row * p.ldres + n0;
          if (full) {
#pragma unroll
            for (int q = 0; q < 4; ++q) {
              const uint4 w = cur[q];
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
        if (row_ok) {
          const __nv_bfloat16* hx = reinterpret_cast<const __nv_bfloat16*>(p.aux) + row * p.ldaux + n0;
          if (full) {
#pragma unroll
            for (int q = 0; q < 4; ++q) {
              const uint4 w = cur[q];
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
      } else if (EPI == kEpiCE) {
        // Statistics use the bf16-rounded logits the backward pass reads back:
        // pairs are packed once (also the stored values) and unpacked.
        constexpr float kLog2e = 1.4426950408889634f;
#pragma unroll
        for (int q = 0; q < 16; ++q) ce_pk[q] = pack_bf16x2(v[2 * q], v[2 * q + 1]);
#pragma unroll
        for (int q = 0; q < 16; ++q) {
          v[2 * q] = __uint_as_float(ce_pk[q] << 16);
          v[2 * q + 1] = __uint_as_float(ce_pk[q] & 0xFFFF0000u);
        }
        float cm = -INFINITY;
        if (full) {
#pragma unroll
          for (int j = 0; j < 32; ++j) cm = fmaxf(cm, v[j]);
        } else {
#pragma unroll
          for (int j = 0; j < 32; ++j)
            if (n0 + j < p.N) cm = fmaxf(cm, v[j]);
        }
        if (cm > ce_m) {
          ce_s = ce_any ? ce_s * ex2_approx((ce_m - cm) * kLog2e) : 0.f;
          ce_m = cm;
        }
        ce_any = true;
        const float mb = ce_m * kLog2e;
        float s = 0.f;
        if (full) {
#pragma unroll
          for (int j = 0; j < 32; ++j) s += ex2_approx(fmaf(v[j], kLog2e, -mb));
        } else {
#pragma unroll
          for (int j = 0; j < 32; ++j)
            if (n0 + j < p.N) s += ex2_approx(fmaf(v[j], kLog2e, -mb));
        }
        ce_s += s;
        if (row_ok && tgt >= n0 && tgt < n0 + 32) {
          float tv = 0.f;
#pragma unroll
          for (int j = 0; j < 32; ++j)
            if (n0 + j == tgt) tv = v[j];
          p.ce_tgt[row] = tv;
        }
      }

      // Stage and write out.
      if (kF32) {
        sb = slab_acquire(es);
#pragma unroll
        for (int k = 0; k < 8; ++k)
          asm volatile("st.shared.v4.f32 [%0], {%1, %2, %3, %4};" ::"r"(smem_u32(sb + sw128_off(lane, k))),
                       "f"(v[4 * k]), "f"(v[4 * k + 1]), "f"(v[4 * k + 2]), "f"(v[4 * k + 3])
                       : "memory");
        slab_issue(es, tmD, sb, f32_mode, to_ws ? 3 : 2, n0, row0, split);
      } else {
        const bool two = EPI == kEpiBF16 && p.gelu;  // output + pre-activation slabs (four epilogue warps)
        if ((c & 1) == 0 && !two) sb = slab_acquire(es);
        if (EPI == kEpiCE) {  // already packed
#pragma unroll
          for (int q = 0; q < 4; ++q)
            asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(
                             smem_u32(sb + sw128_off(lane, (c & 1) * 4 + q))),
                         "r"(ce_pk[4 * q]), "r"(ce_pk[4 * q + 1]), "r"(ce_pk[4 * q + 2]), "r"(ce_pk[4 * q + 3])
                         : "memory");
        } else {
#pragma unroll
          for (int q = 0; q < 4; ++q)
            asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(
                             smem_u32(sb + sw128_off(lane, (c & 1) * 4 + q))),
                         "r"(pack_bf16x2(v[q * 8 + 0], v[q * 8 + 1])), "r"(pack_bf16x2(v[q * 8 + 2], v[q * 8 + 3])),
                         "r"(pack_bf16x2(v[q * 8 + 4], v[q * 8 + 5])), "r"(pack_bf16x2(v[q * 8 + 6], v[q * 8 + 7]))
                         : "memory");
        }
        if ((c & 1) == 1 || n0 + 32 >= p.N) {
          if (EPI == kEpiDGELU && p.colsum != nullptr && row0 < p.M) {  // warp-uniform
            // Bias-gradient first stage from the staged bf16 slab (32 rows x 64
            // columns): lane l sums columns 2l, 2l+1 down the rows, one
            // conflict-free 128-byte row per load.
            __syncwarp();
            const int sn0 = n0 - (c & 1) * 32;
            const int rows = min(32, p.M - row0);
            float s0 = 0.f, s1 = 0.f;
#pragma unroll 8
            for (int r = 0; r < rows; ++r) {
              uint32_t w;
              asm volatile("ld.shared.b32 %0, [%1];"
                           : "=r"(w)
                           : "r"(smem_u32(sb + sw128_off(r, lane >> 2)) + (lane & 3) * 4));
              const float2 f = unpack_bf16x2(w);
              s0 += f.x;
              s1 += f.y;
            }
            float* dst = p.colsum + static_cast<long long>(row0 >> 5) * p.N;
            if (sn0 + 2 * lane < p.N) dst[sn0 + 2 * lane] = s0;
            if (sn0 + 2 * lane + 1 < p.N) dst[sn0 + 2 * lane + 1] = s1;
          }
          slab_issue(es, tmD, sb, 0, 2, n0 - (c & 1) * 32, row0, 0);
          if (two) slab_issue(es, tmX, es.base + kSlabBytes, 0, 2, n0 - (c & 1) * 32, row0, 0);
        }
      }
    }
    if (EPI == kEpiCE && row_ok) {
      const long long sl = static_cast<long long>(tn) * (BN / kCeSlab) + slab;
      if (sl * kCeSlab < p.N) {
        p.ce_max[sl * p.M + row] = ce_m;
        p.ce_sum[sl * p.M + row] = ce_s;
      }
    }
  }
}

// Peer-wait counters of the fused all-reduce (analysis; off unless
// md_gemm_ar_wait_enable(1)): {CTA run ns, comm-warp ns spent waiting on peer
// flags, launches}.
__device__ int g_gar_pw_on;
__device__ unsigned long long g_gar_pw[3];

// Analysis trace of the fused all-reduce: CTA 0 stamps %globaltimer at its
// hand-offs (no-op unless a trace buffer is passed).
#define MD_AR_TRACE(ar, idx, slot)                                                          \
  do {                                                                                      \
    if ((ar).trace != nullptr && blockIdx.x == 0 && (idx) < 64) (ar).trace[(idx) * 8 + (slot)] = globaltimer_ns(); \
  } while (0)

// ---------------------------------------------------------------------------
// Peer flags for the fused all-reduce
// ---------------------------------------------------------------------------
// Publishing protocol.  Everything a flag publishes (the partial tile, the
// final chunk) and the flag itself live in the publishing GPU's own memory, and
// peers read both over NVLink through that GPU's L2.  The writer therefore
// releases at GPU scope (a system-scope release costs ~10 us here while the
// SM has NVLink traffic in flight); the reader polls the peer flag with
// relaxed system-scope loads and, once it has seen the epoch, orders its
// subsequent loads after that observation with an acquire fence.
__device__ __forceinline__ void flag_release_sys(unsigned* f, unsigned v) {
  asm volatile("st.release.gpu.global.u32 [%0], %1;" ::"l"(f), "r"(v) : "memory");
}
__device__ __forceinline__ unsigned flag_acquire_sys(const unsigned* f) {
  unsigned v;
  asm volatile("ld.relaxed.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(f) : "memory");
  return v;
}
__device__ __forceinline__ void acquire_fence() { asm volatile("fence.acq_rel.gpu;" ::: "memory"); }
// Bounded wait until *f >= v (epochs only grow).  False on timeout / abort.
__device__ __forceinline__ bool flag_wait_ge(const unsigned* f, unsigned v, const MdTpArParams& ar, Status* st,
                                             uint32_t where, volatile int* abort_flag) {
  if (flag_acquire_sys(f) >= v) {
    acquire_fence();
    return true;
  }
  const uint64_t t0 = globaltimer_ns();
  for (uint32_t it = 0;; ++it) {
    if (flag_acquire_sys(f) >= v) {
      acquire_fence();
      return true;
    }
    if ((it & 15u) == 15u) {
      if (*abort_flag) return false;
      if (globaltimer_ns() - t0 > ar.timeout_ns) {
        report(st, kTimeoutPeer, where, v);
        *abort_flag = 1;
        return false;
      }
    }
  }
}

// Comm warp, owned chunk: sum the 32 x 256 chunk over all ranks' partial
// buffers (fixed rank order, so every rank's copy is bit-identical), add bias
// and residual, write the local output and this rank's final buffer, publish.
// Lane l covers columns [8l, 8l+8) of the tile; each step issues the peer
// loads of 16 / W rows for all W ranks at once (16 loads in flight per lane).
template <int W>
__device__ __forceinline__ void ar_reduce_rows(const MdGemmParams& p, const MdTpArParams& ar, int row0, int col,
                                               const float (&bias8)[8]) {
  constexpr int R = 16 / W;  // rows per step
#pragma unroll 1
  for (int i0 = 0; i0 < 32; i0 += R) {
    bool rv[R];
#pragma unroll
    for (int k = 0; k < R; ++k) rv[k] = row0 + i0 + k < p.M;
    uint4 v[R][W];
#pragma unroll
    for (int k = 0; k < R; ++k)
#pragma unroll
      for (int r = 0; r < W; ++r)
        v[k][r] = rv[k] ? __ldcg(reinterpret_cast<const uint4*>(reinterpret_cast<const __nv_bfloat16*>(ar.partial[r]) +
                                                               (row0 + i0 + k) * ar.ldp + col))
                        : make_uint4(0, 0, 0, 0);
    uint4 rs[R];
#pragma unroll
    for (int k = 0; k < R; ++k)
      rs[k] = (ar.resid != nullptr && rv[k])
                  ? *reinterpret_cast<const uint4*>(reinterpret_cast<const __nv_bfloat16*>(ar.resid) +
                                                    (row0 + i0 + k) * ar.ldr + col)
                  : make_uint4(0, 0, 0, 0);
#pragma unroll
    for (int k = 0; k < R; ++k) {
      if (!rv[k]) continue;
      float acc[8];
#pragma unroll
      for (int j = 0; j < 8; ++j) acc[j] = bias8[j];
#pragma unroll
      for (int r = 0; r < W; ++r) {
        const float2 a = unpack_bf16x2(v[k][r].x), b = unpack_bf16x2(v[k][r].y), c = unpack_bf16x2(v[k][r].z),
                     d = unpack_bf16x2(v[k][r].w);
        acc[0] += a.x; acc[1] += a.y; acc[2] += b.x; acc[3] += b.y;
        acc[4] += c.x; acc[5] += c.y; acc[6] += d.x; acc[7] += d.y;
      }
      {
        const float2 a = unpack_bf16x2(rs[k].x), b = unpack_bf16x2(rs[k].y), c = unpack_bf16x2(rs[k].z),
                     d = unpack_bf16x2(rs[k].w);
        acc[0] += a.x; acc[1] += a.y; acc[2] += b.x; acc[3] += b.y;
        acc[4] += c.x; acc[5] += c.y; acc[6] += d.x; acc[7] += d.y;
      }
      const long long row = row0 + i0 + k;
      uint4 o;
      o.x = pack_bf16x2(acc[0], acc[1]);
      o.y = pack_bf16x2(acc[2], acc[3]);
      o.z = pack_bf16x2(acc[4], acc[5]);
      o.w = pack_bf16x2(acc[6], acc[7]);
      *reinterpret_cast<uint4*>(reinterpret_cast<__nv_bfloat16*>(ar.out) + row * ar.ldo + col) = o;
      __stcg(reinterpret_cast<uint4*>(reinterpret_cast<__nv_bfloat16*>(ar.fin[ar.rank]) + row * ar.ldp + col), o);
    }
  }
}

__device__ __forceinline__ bool ar_reduce_chunk(const MdGemmParams& p, const MdTpArParams& ar, unsigned epoch, int chunk,
                                                int row0, int col0, int lane, volatile int* abort_flag) {
  bool ok = true;
  const uint64_t tw = g_gar_pw_on ? globaltimer_ns() : 0ull;
  if (lane < ar.world) ok = flag_wait_ge(ar.flags[lane] + chunk, epoch, ar, p.status, 60, abort_flag);
  if (__any_sync(0xFFFFFFFFu, !ok)) return false;
  if (tw != 0ull && lane == 0) atomicAdd(&g_gar_pw[1], globaltimer_ns() - tw);
  acquire_fence();  // every lane's loads below follow the lanes' observations (ordered by the vote)
  const int col = col0 + lane * 8;
  if (col < p.N) {
    float bias8[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) bias8[j] = ar.bias != nullptr ? ar.bias[col + j] : 0.f;
    switch (ar.world) {
      case 1: ar_reduce_rows<1>(p, ar, row0, col, bias8); break;
      case 2: ar_reduce_rows<2>(p, ar, row0, col, bias8); break;
      case 4: ar_reduce_rows<4>(p, ar, row0, col, bias8); break;
      default: ar_reduce_rows<8>(p, ar, row0, col, bias8); break;  // md_gemm_ar admits 1, 2, 4, 8 only
    }
  }
  // __syncwarp orders every lane's stores before lane 0's release (which is
  // cumulative), so one release store publishes the whole chunk.
  __syncwarp();
  if (lane == 0) flag_release_sys(ar.flags[ar.rank] + ar.max_chunks + chunk, epoch);
  return true;
}

// Comm warp, chunk owned by `owner`: copy its final values into the output.
// blocking = false returns false at once if the owner has not published yet.
__device__ __forceinline__ int ar_pull_chunk(const MdGemmParams& p, const MdTpArParams& ar, unsigned epoch, int chunk,
                                             int owner, int row0, int col0, int lane, bool blocking,
                                             volatile int* abort_flag) {
  const unsigned* f = ar.flags[owner] + ar.max_chunks + chunk;
  int ready = 0;
  if (lane == 0) {
    if (blocking) {
      const uint64_t tw = g_gar_pw_on ? globaltimer_ns() : 0ull;
      ready = flag_wait_ge(f, epoch, ar, p.status, 61, abort_flag) ? 1 : -1;
      if (tw != 0ull) atomicAdd(&g_gar_pw[1], globaltimer_ns() - tw);
    } else {
      ready = flag_acquire_sys(f) >= epoch ? 1 : 0;
    }
  }
  ready = __shfl_sync(0xFFFFFFFFu, ready, 0);
  if (ready == 1) acquire_fence();  // every lane's loads below follow the observation
  if (ready != 1) return ready;
  const int col = col0 + lane * 8;
  if (col < p.N) {
    const __nv_bfloat16* src = reinterpret_cast<const __nv_bfloat16*>(ar.fin[owner]);
    __nv_bfloat16* dst = reinterpret_cast<__nv_bfloat16*>(ar.out);
    // Sixteen rows of peer loads in flight per step.
#pragma unroll 1
    for (int i0 = 0; i0 < 32; i0 += 16) {
      uint4 v[16];
#pragma unroll
      for (int k = 0; k < 16; ++k) {
        const long long row = row0 + i0 + k;
        v[k] = row < p.M ? __ldcg(reinterpret_cast<const uint4*>(src + row * ar.ldp + col)) : make_uint4(0, 0, 0, 0);
      }
#pragma unroll
      for (int k = 0; k < 16; ++k) {
        const long long row = row0 + i0 + k;
        if (row < p.M) *reinterpret_cast<uint4*>(dst + row * ar.ldo + col) = v[k];
      }
    }
  }
  return 1;
}

// ---------------------------------------------------------------------------
// The kernel
// ---------------------------------------------------------------------------
// The kernel body; gemm_kernel (plain GEMM) and md_gemm_ar_kernel (GEMM +
// tensor-parallel all-reduce: its own name, so profiles attribute it as a
// collective) are its two entry points.  The tensor maps stay in kernel
// parameter space (references to the __grid_constant__ parameters).
template <int CG, int EW, bool A_MN, bool B_MN, int EPI, bool AR>
__device__ __forceinline__ void gemm_body(const CUtensorMap& tmA, const CUtensorMap& tmB, const CUtensorMap& tmD,
                                          const CUtensorMap& tmX, const KParams& kp) {
  using C = Cfg<CG, EW>;
  constexpr int kStages = C::kStages;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sA = smem;
  uint8_t* sB = smem + kStages * kABytes;
  uint8_t* sEpi = smem + kStages * C::kStageBytes;
  uint64_t* bars = reinterpret_cast<uint64_t*>(sEpi + C::kEpiSmem);
  uint64_t* full_bar = bars;
  uint64_t* empty_bar = bars + kStages;
  uint64_t* tfull_bar = bars + 2 * kStages;
  uint64_t* tempty_bar = bars + 2 * kStages + 2;
  uint64_t* drain_bar = bars + 2 * kStages + 4;
  uint32_t* tmem_base_slot = reinterpret_cast<uint32_t*>(bars + 2 * kStages + 5);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(bars + 2 * kStages + 6);
  int* vcid_slot = reinterpret_cast<int*>(bars + 2 * kStages + 7);

  const MdGemmParams& p = kp.p;
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint64_t t_entry = (AR && threadIdx.x == 0 && g_gar_pw_on) ? globaltimer_ns() : 0ull;
  const uint32_t crank = CG == 2 ? cluster_ctarank() : 0u;
  const bool leader = crank == 0;
  int cluster_id = CG == 2 ? static_cast<int>(blockIdx.x >> 1) : static_cast<int>(blockIdx.x);
  const int nclusters = CG == 2 ? static_cast<int>(gridDim.x >> 1) : static_cast<int>(gridDim.x);

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&full_bar[s], 1);
      mbar_init(&empty_bar[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&tfull_bar[a], 1);
      mbar_init(&tempty_bar[a], CG * EW);
    }
    mbar_init(drain_bar, 1);
    *abort_flag = 0;
    if constexpr (AR) {
      if (kp.ar.claim != nullptr && leader) {
        const unsigned v = atomicAdd(kp.ar.claim, 1u);
        *vcid_slot = v < static_cast<unsigned>(nclusters) ? static_cast<int>(v) : nclusters;
        if (v >= static_cast<unsigned>(nclusters)) report(p.status, kTimeoutPeer, 49, v);
        // Launch count of this communicator + 1: the epoch, kept on the device
        // so that a replayed CUDA graph advances it.
        vcid_slot[1] = static_cast<int>(*reinterpret_cast<volatile unsigned*>(kp.ar.claim + 2) + 1u);
      }
    }
    fence_mbar_init();
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
    tma_prefetch_desc(&tmD);
  }
  if (warp == 1) {
    if constexpr (CG == 2) {
      tmem_alloc_pair(tmem_base_slot, kTmemCols);
      tmem_relinquish_pair();
    } else {
      tmem_alloc(tmem_base_slot, kTmemCols);
      tmem_relinquish();
    }
  }
  tc_fence_before();
  __syncthreads();
  if constexpr (CG == 2) cluster_sync();  // peer barriers exist before any cross-CTA arrival
  tc_fence_after();
  const uint32_t tmem_base = *tmem_base_slot;
  if constexpr (!AR) {
    // Prologue done (barriers, TMEM): let the next kernel launch, then wait
    // for the previous one before touching global memory.
    pdl_trigger();
    pdl_wait();
  }
  unsigned ar_epoch = 0;
  if constexpr (AR) {
    ar_epoch = kp.ar.epoch;
    if (kp.ar.claim != nullptr) {
      if constexpr (CG == 2) {
        // The follower reads the leader's claim (written before the cluster barrier).
        uint32_t v, e;
        const uint32_t a = map_to_cta(smem_u32(vcid_slot), 0);
        asm volatile("ld.shared::cluster.u32 %0, [%1];" : "=r"(v) : "r"(a) : "memory");
        asm volatile("ld.shared::cluster.u32 %0, [%1];" : "=r"(e) : "r"(a + 4u) : "memory");
        cluster_id = static_cast<int>(v);
        ar_epoch = e;
      } else {
        cluster_id = vcid_slot[0];
        ar_epoch = static_cast<unsigned>(vcid_slot[1]);
      }
    }
  }

  if (warp == 0 && lane == 0) {
    // ------------------------------------------------------------ producer
    int stage = 0;
    uint32_t phase = 0;
    long long fills = 0;
    int armed_phase[kStages];
    for (int s = 0; s < kStages; ++s) armed_phase[s] = -1;
    bool ok = true;
    for (int u = cluster_id; u < kp.units && ok; u += nclusters) {
      int tm, tn, split;
      decode_unit(kp, u, tm, tn, split);
      const int kb0 = split * kp.kb_per_split;
      const int kb1 = min(kp.k_blocks, kb0 + kp.kb_per_split);
      const int row_base = tm * (CG * BM) + static_cast<int>(crank) * BM;
      const int col_base = tn * BN + static_cast<int>(crank) * (BN / CG);
      for (int kb = kb0; kb < kb1; ++kb) {
        if (!mbar_wait(&empty_bar[stage], phase ^ 1u, p.status, 10, abort_flag)) {
          ok = false;
          break;
        }
        uint32_t bar_addr = smem_u32(&full_bar[stage]);
        if constexpr (CG == 2) {
          bar_addr = map_to_cta(bar_addr, 0);
          if (leader) mbar_arrive_expect_tx(&full_bar[stage], CG * C::kStageBytes);
        } else {
          mbar_arrive_expect_tx(&full_bar[stage], C::kStageBytes);
        }
        armed_phase[stage] = static_cast<int>(phase);
        uint8_t* a_dst = sA + stage * kABytes;
        uint8_t* b_dst = sB + stage * C::kBBytes;
        if (!A_MN) {
          if (CG == 2) tma_load_2d_pair(&tmA, bar_addr, a_dst, kb * BK, row_base);
          else tma_load_2d(&tmA, &full_bar[stage], a_dst, kb * BK, row_base);
        } else {
#pragma unroll
          for (int c = 0; c < BM / 64; ++c) {
            if (CG == 2) tma_load_2d_pair(&tmA, bar_addr, a_dst + c * (64 * BK * 2), row_base + c * 64, kb * BK);
            else tma_load_2d(&tmA, &full_bar[stage], a_dst + c * (64 * BK * 2), row_base + c * 64, kb * BK);
          }
        }
        if (!B_MN) {
          if (CG == 2) tma_load_2d_pair(&tmB, bar_addr, b_dst, kb * BK, col_base);
          else tma_load_2d(&tmB, &full_bar[stage], b_dst, kb * BK, col_base);
        } else {
#pragma unroll
          for (int c = 0; c < (BN / CG) / 64; ++c) {
            if (CG == 2) tma_load_2d_pair(&tmB, bar_addr, b_dst + c * (64 * BK * 2), col_base + c * 64, kb * BK);
            else tma_load_2d(&tmB, &full_bar[stage], b_dst + c * (64 * BK * 2), col_base + c * 64, kb * BK);
          }
        }
        ++fills;
        if (++stage == kStages) {
          stage = 0;
          phase ^= 1u;
        }
      }
    }
    // No bulk copy into shared memory may still be in flight at exit.  (The
    // follower's copies complete on the leader's barriers, which the leader's
    // MMA has consumed before the final cluster barrier.)
    if (CG == 1 || leader)
      for (int s = 0; s < kStages; ++s)
        if (armed_phase[s] >= 0) mbar_wait(&full_bar[s], static_cast<uint32_t>(armed_phase[s]), p.status, 11, nullptr);
  } else if (warp == 1 && leader) {
    // ------------------------------------------------------------ MMA issuer (whole warp, elected lane issues)
    constexpr uint32_t idesc = idesc_bf16_f32(CG * BM, BN, A_MN, B_MN);
    constexpr uint32_t kBChunkStride = 64 * BK * 2;
    // Base descriptors of stage 0; stage s and k-step k are constant byte
    // offsets, added as (offset >> 4).
    const uint64_t a_base = A_MN ? sdesc_sw128(smem_u32(sA), kBChunkStride, 1024) : sdesc_sw128(smem_u32(sA), 16, 1024);
    const uint64_t b_base =
        B_MN ? sdesc_sw128(smem_u32(sB), kBChunkStride, 1024) : sdesc_sw128(smem_u32(sB), 16, 1024);
    int stage = 0;
    uint32_t phase = 0;
    int acc = 0;
    uint32_t acc_phase = 0;
    bool ok = true;
    for (int u = cluster_id; u < kp.units && ok; u += nclusters) {
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
        const uint64_t a_st = a_base + static_cast<uint32_t>(stage * kABytes >> 4);
        const uint64_t b_st = b_base + static_cast<uint32_t>(stage * C::kBBytes >> 4);
#pragma unroll
        for (int k = 0; k < BK / 16; ++k) {
          const uint32_t a_off = A_MN ? k * (2048 >> 4) : k * (32 >> 4);
          const uint32_t b_off = B_MN ? k * (2048 >> 4) : k * (32 >> 4);
          const uint32_t accum = (kb > kb0 || k > 0) ? 1u : 0u;
          umma_elect<CG>(d_tmem, a_st + a_off, b_st + b_off, idesc, accum);
        }
        commit_all_elect<CG>(&empty_bar[stage]);
        if (++stage == kStages) {
          stage = 0;
          phase ^= 1u;
        }
      }
      if (!ok) break;
      commit_all_elect<CG>(&tfull_bar[acc]);
      if (++acc == 2) {
        acc = 0;
        acc_phase ^= 1u;
      }
    }
    // Drain: every MMA this warp issued completes before TMEM is released.
    commit_self_elect<CG>(drain_bar);
    mbar_wait(drain_bar, 0, p.status, 22, nullptr);
  } else if (warp >= 2 && warp < 2 + EW) {
    // ------------------------------------------------------------ epilogue
    const int ew = warp - 2;
    const int quarter = warp & 3;  // TMEM lane quarter this warp may access
    const int c_begin = EW == 8 ? (ew / 4) * 4 : 0;
    const int c_end = EW == 8 ? c_begin + 4 : 8;
    uint32_t tempty_addr[2] = {smem_u32(&tempty_bar[0]), smem_u32(&tempty_bar[1])};
    if constexpr (CG == 2) {
      tempty_addr[0] = map_to_cta(tempty_addr[0], 0);
      tempty_addr[1] = map_to_cta(tempty_addr[1], 0);
    }
    EpiStage es;
    es.nbuf = 2;
    es.base = sEpi + ew * 2 * kSlabBytes;
    es.ctr = 0;
    es.lane = lane;
    int acc = 0;
    uint32_t acc_phase = 0;
    // The epilogue's second input (pre-activation, residual or dot operand) is
    // streamed from HBM one chunk ahead; an L2 prefetch of this thread's row
    // segment of the NEXT tile gives those loads a whole tile of lead time.
    const __nv_bfloat16* pf_base = nullptr;
    long long pf_ld = 0;
    if (EPI == kEpiDGELU) {
      pf_base = reinterpret_cast<const __nv_bfloat16*>(p.aux);
      pf_ld = p.ldaux;
    } else if (EPI == kEpiBF16 && p.resid != nullptr) {
      pf_base = reinterpret_cast<const __nv_bfloat16*>(p.resid);
      pf_ld = p.ldres;
    } else if (EPI == kEpiBF16 && p.dot_out != nullptr) {
      pf_base = reinterpret_cast<const __nv_bfloat16*>(p.dot_in);
      pf_ld = p.lddot;
    }
    auto prefetch_in = [&](int uu) {
      if (pf_base == nullptr || uu >= kp.units) return;
      int tm2, tn2, sp2;
      decode_unit(kp, uu, tm2, tn2, sp2);
      const long long row = tm2 * (CG * BM) + static_cast<int>(crank) * BM + quarter * 32 + lane;
      const int col0 = tn2 * BN + c_begin * 32;
      const int col1 = min(p.N, tn2 * BN + c_end * 32);
      if (row >= p.M || col0 >= col1) return;
      const char* a = reinterpret_cast<const char*>(pf_base + row * pf_ld + col0);
      const char* e = reinterpret_cast<const char*>(pf_base + row * pf_ld + col1) - 1;
      for (const char* q = a; q < e; q += 128) asm volatile("prefetch.global.L2 [%0];" ::"l"(q));
      asm volatile("prefetch.global.L2 [%0];" ::"l"(e));
    };
    prefetch_in(cluster_id);
    for (int u = cluster_id; u < kp.units; u += nclusters) {
      int tm, tn, split;
      decode_unit(kp, u, tm, tn, split);
      prefetch_in(u + nclusters);
      if (!mbar_wait(&tfull_bar[acc], acc_phase, p.status, 30, abort_flag)) break;
      tc_fence_after();
      const int row0 = tm * (CG * BM) + static_cast<int>(crank) * BM + quarter * 32;
      const uint32_t t_row =
          tmem_base + (static_cast<uint32_t>(quarter * 32) << 16) + static_cast<uint32_t>(acc * BN);
      epilogue_row<EPI>(p, &tmD, &tmX, es, row0 + lane, row0, tn, split, t_row, c_begin, c_end);
      if constexpr (AR) {
        // Publish this chunk of the partial product once its bulk stores have
        // completed (bulk-async writes, then a proxy fence, then the release).
        if (lane == 0 && row0 < p.M) {
          const int ti = (u - cluster_id) / nclusters;
          if (quarter == 0) MD_AR_TRACE(kp.ar, ti, 0);
          bulk_wait_all();
          if (quarter == 0) MD_AR_TRACE(kp.ar, ti, 7);
          // The completed bulk writes are ordered before the release by the
          // proxy fence; the release store itself publishes them system-wide.
          asm volatile("fence.proxy.async.global;" ::: "memory");
          if (quarter == 0) MD_AR_TRACE(kp.ar, ti, 6);
          flag_release_sys(kp.ar.flags[kp.ar.rank] + (row0 >> 5) * kp.tiles_n + tn, ar_epoch);
          if (quarter == 0) MD_AR_TRACE(kp.ar, ti, 1);
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) {
        if constexpr (CG == 2) mbar_arrive_remote(tempty_addr[acc]);
        else mbar_arrive(&tempty_bar[acc]);
      }
      if (++acc == 2) {
        acc = 0;
        acc_phase ^= 1u;
      }
    }
    // Every bulk store / reduce-add of this warp has completed before exit.
    if (lane == 0) bulk_wait_all();
  } else if (AR && warp >= 2 + EW) {
    // ------------------------------------------------------------ all-reduce (comm warps)
    // Same tile walk as the epilogue; this warp covers the 32 rows of one
    // lane quarter.  Owned chunks are reduced as soon as every rank has
    // published its partial; the others are copied from their owners, first
    // opportunistically in between, then (blocking) at the end.
    const MdTpArParams& ar = kp.ar;
    const int quarter = warp & 3;
    int pull_u = cluster_id;  // next tile whose non-owned chunk still has to be copied
    bool ok = true;
    auto chunk_of = [&](int u, int& row0, int& col0, int& chunk) {
      int tm, tn, split;
      decode_unit(kp, u, tm, tn, split);
      row0 = tm * (CG * BM) + static_cast<int>(crank) * BM + quarter * 32;
      col0 = tn * BN;
      chunk = (row0 >> 5) * kp.tiles_n + tn;
    };
    auto try_pulls = [&](int limit_u, bool blocking) {
      while (ok && pull_u < limit_u) {
        int row0, col0, chunk;
        chunk_of(pull_u, row0, col0, chunk);
        const int owner = chunk % ar.world;
        if (row0 < p.M && owner != ar.rank) {
          const int r = ar_pull_chunk(p, ar, ar_epoch, chunk, owner, row0, col0, lane, blocking, abort_flag);
          if (r < 0) ok = false;
          if (r != 1) return;
        }
        pull_u += nclusters;
      }
    };
    for (int u = cluster_id; u < kp.units && ok; u += nclusters) {
      int row0, col0, chunk;
      chunk_of(u, row0, col0, chunk);
      const int ti = (u - cluster_id) / nclusters;
      if (quarter == 0 && lane == 0) MD_AR_TRACE(ar, ti, 2);
      if (row0 < p.M && chunk % ar.world == ar.rank) {
        ok = ar_reduce_chunk(p, ar, ar_epoch, chunk, row0, col0, lane, abort_flag);
        if (quarter == 0 && lane == 0) MD_AR_TRACE(ar, ti, 3);
      }
      try_pulls(u + 1, false);
      if (quarter == 0 && lane == 0) MD_AR_TRACE(ar, ti, 4);
    }
    if (quarter == 0 && lane == 0) MD_AR_TRACE(ar, 63, 5);
    try_pulls(kp.units, true);
    if (quarter == 0 && lane == 0) MD_AR_TRACE(ar, 63, 6);
  }

  tc_fence_before();
  __syncthreads();
  if constexpr (CG == 2) cluster_sync();
  tc_fence_after();
  if (warp == 1) {
    if constexpr (CG == 2) tmem_dealloc_pair(tmem_base, kTmemCols);
    else tmem_dealloc(tmem_base, kTmemCols);
  }
  if constexpr (AR) {
    if (t_entry != 0ull) atomicAdd(&g_gar_pw[0], globaltimer_ns() - t_entry);
    // The launch's last cluster resets the counters for the next launch.
    if (kp.ar.claim != nullptr && leader && threadIdx.x == 0 &&
        atomicAdd(kp.ar.claim + 1, 1u) == static_cast<unsigned>(nclusters - 1)) {
      atomicExch(kp.ar.claim + 2, ar_epoch);
      atomicExch(kp.ar.claim, 0u);
      atomicExch(kp.ar.claim + 1, 0u);
      if (t_entry != 0ull) atomicAdd(&g_gar_pw[2], 1ull);
    }
  }
}

template <int CG, int EW, bool A_MN, bool B_MN, int EPI>
__global__ void __launch_bounds__(64 + 32 * EW, 1)
    gemm_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                const __grid_constant__ CUtensorMap tmD, const __grid_constant__ CUtensorMap tmX,
                const __grid_constant__ KParams kp) {
  gemm_body<CG, EW, A_MN, B_MN, EPI, false>(tmA, tmB, tmD, tmX, kp);
}

template <int CG, int EW, bool A_MN, bool B_MN, int EPI>
__global__ void __launch_bounds__(64 + 32 * EW + 128, 1)
    md_gemm_ar_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                      const __grid_constant__ CUtensorMap tmD, const __grid_constant__ CUtensorMap tmX,
                      const __grid_constant__ KParams kp) {
  gemm_body<CG, EW, A_MN, B_MN, EPI, true>(tmA, tmB, tmD, tmX, kp);
}

template <int CG, int EW, bool A_MN, bool B_MN, int EPI, bool AR>
struct KernelFor {
  static constexpr auto fn = gemm_kernel<CG, EW, A_MN, B_MN, EPI>;
};
template <int CG, int EW, bool A_MN, bool B_MN, int EPI>
struct KernelFor<CG, EW, A_MN, B_MN, EPI, true> {
  static constexpr auto fn = md_gemm_ar_kernel<CG, EW, A_MN, B_MN, EPI>;
};

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

// Output map for the TMA-store epilogue: [depth, outer, inner] (depth 0 = 2-D)
// with 128B swizzle and a box of 128 bytes x 32 rows (64 bf16 / 32 fp32).
bool make_out_map(CUtensorMap* map, void* ptr, bool f32, uint64_t inner, uint64_t outer, uint64_t ld_elems,
                  uint64_t depth) {
  const uint64_t es = f32 ? 4 : 2;
  cuuint64_t dims[3] = {inner, outer, depth};
  cuuint64_t strides[2] = {ld_elems * es, ld_elems * es * outer};
  cuuint32_t box[3] = {static_cast<cuuint32_t>(128 / es), 32, 1};
  cuuint32_t estr[3] = {1, 1, 1};
  const cuuint32_t rank = depth > 0 ? 3 : 2;
  CUresult r = g_encode(map, f32 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, rank, ptr, dims,
                        strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                        CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

int g_num_sms = 0;

template <int CG, int kEW, bool A_MN, bool B_MN, int EPI, bool AR = false>
cudaError_t launch(const CUtensorMap& ta, const CUtensorMap& tb, const CUtensorMap& td, const CUtensorMap& tx,
                   const md::gemm::KParams& kp, int grid, cudaStream_t stream) {
  auto kern = md::gemm::KernelFor<CG, kEW, A_MN, B_MN, EPI, AR>::fn;
  constexpr int smem = md::gemm::Cfg<CG, kEW>::kSmemBytes;
  static int attr_done[64] = {0};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 64 && !attr_done[dev]) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (e != cudaSuccess) return e;
    if (CG == 2) {
      e = cudaFuncSetAttribute(kern, cudaFuncAttributeNonPortableClusterSizeAllowed, 0);
      (void)e;
    }
    attr_done[dev] = 1;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(64 + 32 * kEW + (AR ? 128 : 0));
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[2];
  cfg.attrs = attr;
  cfg.numAttrs = 0;
  if (CG == 2) {
    attr[cfg.numAttrs].id = cudaLaunchAttributeClusterDimension;
    attr[cfg.numAttrs].val.clusterDim.x = 2;
    attr[cfg.numAttrs].val.clusterDim.y = 1;
    attr[cfg.numAttrs].val.clusterDim.z = 1;
    ++cfg.numAttrs;
  }
  // The fused all-reduce variant waits on peers: never launched early next to
  // its predecessor (it keeps plain stream order).
  if (!AR && md::pdl_enabled()) {
    attr[cfg.numAttrs].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[cfg.numAttrs].val.programmaticStreamSerializationAllowed = 1;
    ++cfg.numAttrs;
  }
  return cudaLaunchKernelEx(&cfg, kern, ta, tb, td, tx, kp);
}

template <int CG, int EW>
cudaError_t dispatch(bool amn, bool bmn, int epi, const CUtensorMap& ta, const CUtensorMap& tb, const CUtensorMap& td,
                     const CUtensorMap& tx, const md::gemm::KParams& kp, int grid, cudaStream_t s, bool* bad) {
  using namespace md::gemm;
  *bad = false;
  if (!amn && !bmn) {
    if (epi == kEpiBF16) return launch<CG, EW, false, false, kEpiBF16>(ta, tb, td, tx, kp, grid, s);
    if (epi == kEpiF32) return launch<CG, EW, false, false, kEpiF32>(ta, tb, td, tx, kp, grid, s);
    if (epi == kEpiCE) return launch<CG, EW, false, false, kEpiCE>(ta, tb, td, tx, kp, grid, s);
  } else if (!amn && bmn) {
    if (epi == kEpiBF16) return launch<CG, EW, false, true, kEpiBF16>(ta, tb, td, tx, kp, grid, s);
    if (epi == kEpiF32) return launch<CG, EW, false, true, kEpiF32>(ta, tb, td, tx, kp, grid, s);
    if (epi == kEpiDGELU) return launch<CG, EW, false, true, kEpiDGELU>(ta, tb, td, tx, kp, grid, s);
  } else if (amn && bmn) {
    if (epi == kEpiF32) return launch<CG, EW, true, true, kEpiF32>(ta, tb, td, tx, kp, grid, s);
    if (epi == kEpiBF16) return launch<CG, EW, true, true, kEpiBF16>(ta, tb, td, tx, kp, grid, s);
  } else {
    if (epi == kEpiF32) return launch<CG, EW, true, false, kEpiF32>(ta, tb, td, tx, kp, grid, s);
    if (epi == kEpiBF16) return launch<CG, EW, true, false, kEpiBF16>(ta, tb, td, tx, kp, grid, s);
  }
  *bad = true;
  return cudaSuccess;
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
    if (p.k_splits > 1 && p.workspace != nullptr && (!aligned16(p.workspace) || (p.ldws % 4))) return -6;
  } else {
    if (!aligned16(p.D) || (p.ldd % 8)) return -5;
    if (p.k_splits != 1) return -6;
  }
  if (p.gelu && (p.aux == nullptr || !aligned16(p.aux) || (p.ldaux % 8))) return -7;
  if (p.epi == kEpiDGELU && (p.aux == nullptr || !aligned16(p.aux) || (p.ldaux % 8))) return -7;
  if (p.resid != nullptr && (!aligned16(p.resid) || (p.ldres % 8))) return -8;
  if (p.dot_out != nullptr &&
      (p.epi != kEpiBF16 || p.gelu || p.resid != nullptr || p.k_splits != 1 || p.dot_in == nullptr ||
       !aligned16(p.dot_in) || (p.lddot % 8) || !(p.dot_group == 32 || p.dot_group == 64 || p.dot_group == 128) ||
       (p.N % p.dot_group) || p.dot_seq <= 0 || (p.M % p.dot_seq)))
    return -10;
  if (p.epi == kEpiCE && (p.ce_target == nullptr || p.ce_max == nullptr || p.ce_sum == nullptr || p.ce_tgt == nullptr))
    return -9;
  if (p.k_splits < 1) p.k_splits = 1;

  if (g_num_sms == 0) {
    int dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&g_num_sms, cudaDevAttrMultiProcessorCount, dev);
  }
  // Tile configuration: the 2-CTA 256x256 tiles win whenever there are enough
  // rows; weight-gradient products with few output rows keep 128-row tiles
  // (more tiles to spread over the SMs).
  int cg = p.cta_group;
  if (cg != 1 && cg != 2) cg = p.a_mn_major ? (p.M >= 2304 ? 2 : 1) : (p.M >= 512 ? 2 : 1);
  // Four epilogue warps measured best across the GPT shapes (eight only
  // matched it for the GELU / cross-entropy epilogues).
  // Eight epilogue warps where the epilogue does real work per element and the
  // mainloop is too short to hide it (GELU, dGELU, cross-entropy statistics,
  // residual add with K <= 1024); four (and one more mainloop stage)
  // otherwise.  Measured in the GPT-2 step: fc+GELU 118 -> 97 us, proj+residual
  // (K = 768) 41 -> 34 us; mlp.proj+residual (K = 3072) prefers four.
  if (p.epi_warps != 4 && p.epi_warps != 8)
    p.epi_warps = (p.epi == kEpiCE || p.epi == kEpiDGELU ||
                   (p.epi == kEpiBF16 && (p.gelu || (p.resid && p.K <= 1024)))) ? 8 : 4;

  CUtensorMap ta, tb;
  bool ok;
  if (!p.a_mn_major) ok = make_map(&ta, p.A, p.K, p.M, p.lda, BM);
  else               ok = make_map(&ta, p.A, p.M, p.K, p.lda, 64);
  if (!ok) return -10;
  if (!p.b_mn_major) ok = make_map(&tb, p.B, p.K, p.N, p.ldb, BN / cg);
  else               ok = make_map(&tb, p.B, p.N, p.K, p.ldb, 64);
  if (!ok) return -11;

  KParams kp;
  kp.p = p;
  kp.tiles_m = (p.M + cg * BM - 1) / (cg * BM);
  kp.tiles_n = (p.N + BN - 1) / BN;
  kp.k_blocks = (p.K + BK - 1) / BK;
  if (p.k_splits > kp.k_blocks) p.k_splits = kp.k_blocks;
  kp.kb_per_split = (kp.k_blocks + p.k_splits - 1) / p.k_splits;
  kp.p.k_splits = (kp.k_blocks + kp.kb_per_split - 1) / kp.kb_per_split;  // no empty split
  kp.units = kp.tiles_m * kp.tiles_n * kp.p.k_splits;

  CUtensorMap td;
  if (p.epi == kEpiF32 && kp.p.k_splits > 1 && p.workspace != nullptr)
    ok = make_out_map(&td, p.workspace, true, p.N, p.M, p.ldws, kp.p.k_splits);
  else
    ok = make_out_map(&td, p.D, p.epi == kEpiF32, p.N, p.M, p.ldd, 0);
  if (!ok) return -13;
  CUtensorMap tx = td;  // second epilogue output: the GELU pre-activation
  if (p.epi == kEpiBF16 && p.gelu && !make_out_map(&tx, p.aux, false, p.N, p.M, p.ldaux, 0)) return -14;

  int cap = p.num_sms > 0 ? p.num_sms : g_num_sms;
  int grid;
  if (cg == 2) {
    const int clusters = kp.units < cap / 2 ? kp.units : cap / 2;
    grid = 2 * (clusters > 0 ? clusters : 1);
  } else {
    grid = kp.units < cap ? kp.units : cap;
  }

  if (p.epi == kEpiF32 && kp.p.k_splits > 1 && p.workspace == nullptr && !p.beta) {
    cudaError_t ez = cudaMemset2DAsync(p.D, static_cast<size_t>(p.ldd) * 4, 0, static_cast<size_t>(p.N) * 4,
                                       static_cast<size_t>(p.M), stream);
    if (ez != cudaSuccess) return static_cast<int>(ez);
  }
  bool bad = false;
  const int ew = p.epi_warps == 4 ? 4 : 8;
  cudaError_t e;
  if (cg == 2) {
    e = ew == 4 ? dispatch<2, 4>(p.a_mn_major, p.b_mn_major, p.epi, ta, tb, td, tx, kp, grid, stream, &bad)
                : dispatch<2, 8>(p.a_mn_major, p.b_mn_major, p.epi, ta, tb, td, tx, kp, grid, stream, &bad);
  } else {
    e = ew == 4 ? dispatch<1, 4>(p.a_mn_major, p.b_mn_major, p.epi, ta, tb, td, tx, kp, grid, stream, &bad)
                : dispatch<1, 8>(p.a_mn_major, p.b_mn_major, p.epi, ta, tb, td, tx, kp, grid, stream, &bad);
  }
  if (bad) return -12;
  if (e != cudaSuccess) return static_cast<int>(e);

  if (p.epi == kEpiF32 && kp.p.k_splits > 1 && p.workspace != nullptr) {
    const long long total = static_cast<long long>(p.M) * p.N;
    int blocks = static_cast<int>((total + 255) / 256);
    if (blocks > 32 * g_num_sms) blocks = 32 * g_num_sms;
    md::gemm::splitk_reduce_kernel<<<blocks, 256, 0, stream>>>(p.workspace, reinterpret_cast<float*>(p.D), p.ldd,
                                                               p.ldws, p.M, p.N, kp.p.k_splits, p.beta);
    e = cudaGetLastError();
    if (e != cudaSuccess) return static_cast<int>(e);
  }
  return 0;
}

// 1 when kernels are launched with programmatic dependent launch (MINIDIST_PDL).
extern "C" int md_pdl_enabled() { return md::pdl_enabled() ? 1 : 0; }

// Width of the column slabs the kEpiCE epilogue keeps statistics for.
extern "C" int md_gemm_ce_slab() { return md::gemm::kCeSlab; }

// GEMM + tensor-parallel all-reduce in one kernel (see MdTpArParams):
// out = resid + bias + sum over ranks of (A_r B_r^T), bf16.  A K-major, B
// K-major (forward) or MN-major (data gradient, dx = dy W); plain bf16
// epilogue (alpha only) for the partials; prm->D is ignored (the
// partial goes to ar->partial[ar->rank]).  Every rank of the group calls it
// with the same shapes and epoch.
static unsigned long long* g_ar_trace = nullptr;  // analysis trace buffer (md_gemm_ar_trace_enable)

extern "C" int md_gemm_ar(const MdGemmParams* prm, const MdTpArParams* arp, cudaStream_t stream) {
  using namespace md::gemm;
  if (prm == nullptr || arp == nullptr) return -1;
  MdGemmParams p = *prm;
  const MdTpArParams& ar = *arp;
  if (p.M <= 0 || p.N <= 0 || p.K <= 0) return -2;
  if (!get_encoder()) return -3;
  if (!aligned16(p.A) || !aligned16(p.B) || (p.lda % 8) || (p.ldb % 8)) return -4;
  if (p.a_mn_major || p.epi != kEpiBF16 || p.gelu || p.bias || p.resid || p.k_splits > 1) return -5;
  if ((ar.world != 1 && ar.world != 2 && ar.world != 4 && ar.world != 8) || ar.rank < 0 || ar.rank >= ar.world ||
      (ar.ldp % 8) || (ar.ldo % 8) ||
      (p.N % 8) || !aligned16(ar.out) || (ar.resid != nullptr && (!aligned16(ar.resid) || (ar.ldr % 8))))
    return -6;
  p.D = ar.partial[ar.rank];
  p.ldd = ar.ldp;
  p.k_splits = 1;
  if (g_num_sms == 0) {
    int dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&g_num_sms, cudaDevAttrMultiProcessorCount, dev);
  }
  int cg = p.cta_group;
  if (cg != 1 && cg != 2) cg = p.M >= 512 ? 2 : 1;
  CUtensorMap ta, tb, td;
  if (!make_map(&ta, p.A, p.K, p.M, p.lda, BM)) return -10;
  if (!p.b_mn_major) {
    if (!make_map(&tb, p.B, p.K, p.N, p.ldb, BN / cg)) return -11;
  } else if (!make_map(&tb, p.B, p.N, p.K, p.ldb, 64)) {
    return -11;
  }
  if (!make_out_map(&td, p.D, false, p.N, p.M, p.ldd, 0)) return -13;
  KParams kp;
  kp.p = p;
  kp.tiles_m = (p.M + cg * BM - 1) / (cg * BM);
  kp.tiles_n = (p.N + BN - 1) / BN;
  kp.k_blocks = (p.K + BK - 1) / BK;
  kp.kb_per_split = kp.k_blocks;
  kp.units = kp.tiles_m * kp.tiles_n;
  kp.ar = ar;
  kp.ar.trace = g_ar_trace;
  if (((p.M + 31) / 32) * kp.tiles_n > ar.max_chunks) return -7;
  if (kp.ar.timeout_ns == 0) kp.ar.timeout_ns = 10000000000ull;
  // Every tile's CTA must be resident at once (comm warps wait on peers that
  // wait on the same CTA index), so the grid never exceeds the SM count.
  const int cap = p.num_sms > 0 ? p.num_sms : g_num_sms;
  int grid;
  if (cg == 2) {
    const int clusters = kp.units < cap / 2 ? kp.units : cap / 2;
    grid = 2 * (clusters > 0 ? clusters : 1);
  } else {
    grid = kp.units < cap ? kp.units : cap;
  }
  cudaError_t e;
  if (p.b_mn_major)  // data-gradient products: dx = dy W
    e = cg == 2 ? launch<2, 4, false, true, kEpiBF16, true>(ta, tb, td, td, kp, grid, stream)
                : launch<1, 4, false, true, kEpiBF16, true>(ta, tb, td, td, kp, grid, stream);
  else
    e = cg == 2 ? launch<2, 4, false, false, kEpiBF16, true>(ta, tb, td, td, kp, grid, stream)
                : launch<1, 4, false, false, kEpiBF16, true>(ta, tb, td, td, kp, grid, stream);
  return static_cast<int>(e);
}

// Peer-wait counters of md_gemm_ar: on != 0 turns counting on for the current
// device; reset != 0 zeroes them first.  md_gemm_ar_wait_read copies
// {run_ns, wait_ns, launches} to host memory.  Host-synchronous (analysis only).
extern "C" int md_gemm_ar_wait_enable(int on, int reset) {
  if (reset) {
    unsigned long long zero[3] = {0ull, 0ull, 0ull};
    cudaError_t e = cudaMemcpyToSymbol(md::gemm::g_gar_pw, zero, sizeof(zero));
    if (e != cudaSuccess) return static_cast<int>(e);
  }
  return static_cast<int>(cudaMemcpyToSymbol(md::gemm::g_gar_pw_on, &on, sizeof(int)));
}
extern "C" int md_gemm_ar_wait_read(unsigned long long* out) {
  return static_cast<int>(cudaMemcpyFromSymbol(out, md::gemm::g_gar_pw, sizeof(md::gemm::g_gar_pw)));
}

// Analysis: allocate (enable=1) / free (enable=0) the md_gemm_ar trace buffer;
// md_gemm_ar_trace_read copies its [64][8] stamps to host memory.
extern "C" int md_gemm_ar_trace_enable(int enable) {
  if (enable && g_ar_trace == nullptr) {
    if (cudaMalloc(&g_ar_trace, 64 * 8 * 8) != cudaSuccess) return -1;
    cudaMemset(g_ar_trace, 0, 64 * 8 * 8);
  } else if (!enable && g_ar_trace != nullptr) {
    cudaFree(g_ar_trace);
    g_ar_trace = nullptr;
  }
  return 0;
}
extern "C" int md_gemm_ar_trace_read(unsigned long long* host) {
  if (g_ar_trace == nullptr) return -1;
  return static_cast<int>(cudaMemcpy(host, g_ar_trace, 64 * 8 * 8, cudaMemcpyDeviceToHost));
}
