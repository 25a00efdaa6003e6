// Causal flash attention forward on the 5th-generation tensor cores (tcgen05),
// bf16 in / bf16 out, head_dim 64 or 128 (80 on zero-padded 128 boxes).
//
// Same contract as md_attn_fwd of attention.cu (which dispatches here for
// these head sizes): Q, K, V are read in place from the QKV projection output
// [B*S, ldq] whose columns are interleaved per head as [H, 3, D] (reference
// models/gpt.py:92-99, 123-126: F.scaled_dot_product_attention(is_causal=True));
// the output is [B*S, ldo] with head h at columns h*D; lse [B, H, S] holds the
// natural-log log-sum-exp of every query row for the backward pass.
//
// Persistent kernel (two CTAs per SM for head_dim 64, one for 128), warp-specialised:
//   warp 0      TMA: Q tiles (128 queries, two buffers: the next work item's Q
//               loads while this one runs) and, per key block, K and V tiles
//               (128 keys) through a 3-D tensor map [B, S, 3*H*D] whose
//               sequence-end rows read as zero.  It also stores each finished
//               item's output tile, which the softmax warps stage in that
//               item's (no longer needed) Q buffer, with a bulk tensor store,
//               and reloads the buffer once the store has read it.
//   warp 1      MMA issuer (one thread): S = Q K^T into a TMEM score buffer
//               (128 x 128 fp32; two buffers for head_dim 128), then O += P V
//               into a TMEM accumulator (128 x D fp32) with P read from TMEM.
//               The score product of block g+1 is queued before the P V
//               product of block g (the softmax warps release the score buffer
//               as soon as it is in registers), so the tensor core computes
//               scores while the softmax warps exponentiate.
//   warps 2..   softmax: thread t owns query row t (TMEM lane t, 32x32b loads);
//               for head_dim 128 two warps share each row (keys 0..63 /
//               64..127) and exchange row maxima and sums through shared
//               memory.  Scores come out of TMEM, exp2 on the MUFU pipe, P goes
//               back to TMEM as bf16 pairs (the A operand of P V: no shared-
//               memory round trip, no proxy fence).  The running max only moves
//               when it grows by more than 2^8 (factor kRescaleLog2), so the O
//               rescale (TMEM load/scale/store) is rare after the first blocks;
//               l and O stay consistent since both use the same stale max.
//               The epilogue writes O / l into the 128B-swizzled staging tile
//               and lse straight to global memory, then moves on to the next
//               item while warp 0 stores the tile.
//
// Work items are (query tile, batch*head) pairs ordered longest-first (the
// causal tile qt has qt+1 key blocks) and dealt round-robin to the CTAs.
//
// Every mbarrier wait is bounded (md_sm100.cuh); a CTA that gives up records a
// status, lets the other roles see the abort flag, drains its bulk copies and
// MMAs, frees TMEM and exits.

#include <cudaTypedefs.h>
#include <stdlib.h>

#include "md_sm100.cuh"

namespace md {
namespace attn_tc {

constexpr int kBM = 128;   // queries per tile (TMEM lanes)
constexpr int kBN = 128;   // keys per block
constexpr float kRescaleLog2 = 8.0f;

// head_dim 64 runs two CTAs per SM (96 KB shared memory, 256 TMEM columns
// each) so two independent softmax pipelines share every SM sub-partition and
// hide each other's latencies.  head_dim 128 needs one SM per CTA; there each
// query row is split over two softmax warps (key columns 0..63 and 64..127,
// row maxima and sums exchanged through shared memory) so that every SM
// sub-partition still runs two softmax warps.
template <int D>
struct FwdCfg {
  static constexpr int kChunks = D / 64;               // 64-column (128 B) swizzle atoms along head_dim
  static constexpr int kTileBytes = kBM * D * 2;       // one Q/K/V (or staged O) tile
  static constexpr int kCtasPerSm = D == 64 ? 2 : 1;
  static constexpr int kSplit = D == 64 ? 1 : 2;       // softmax warps per query row
  static constexpr int kSoftWarps = 4 * kSplit;
  static constexpr int kThreads = 64 + 32 * kSoftWarps;
  static constexpr int kQBufs = 2;
  static constexpr int kKvStages = 2;
  static constexpr int kSBufs = D == 64 ? 1 : 2;       // TMEM score buffers
  static constexpr int kRedBytes = kSplit == 2 ? 2 * 2 * kBM * 4 : 0;  // row exchange [parity][half][row] fp32
  static constexpr int kBarBytes = kSplit == 2 ? 512 : 256;
  static constexpr int kSmemData = (kQBufs + 2 * kKvStages) * kTileBytes + kRedBytes;
  static constexpr int kSmemBytes = kSmemData + kBarBytes + 1024 /*alignment slack*/;
  // TMEM: score buffers, then O (D columns), then P (128 keys as bf16 pairs: 64 columns).
  static constexpr uint32_t kTmemCols = D == 64 ? 256 : 512;
  static constexpr uint32_t kOCol = kSBufs * 128;
  static constexpr uint32_t kPCol = kOCol + D;
  // P buffers: two where TMEM has room (head_dim 128), so block g+1's P is written
  // while P V of block g still reads block g's.
  static constexpr int kPBufs = D == 64 ? 1 : 2;
  static_assert(kPCol + kPBufs * kBN / 2 <= kTmemCols, "TMEM columns");
};

struct FwdParams {
  float* lse;
  int B, H, S;
  int n_qt;       // query tiles per sequence
  int items;      // n_qt * B * H
  float scale_log2;
  Status* status;
  // Real head dimension dr <= D.  dr < D (d = 80 on the D = 128 kernel): the
  // tensor maps are 4-D [B, S, head slots, dr], so the 64-column boxes read
  // zeros past dr (they add nothing to QK^T or PV) and the output store
  // clips columns past dr.
  int dr;
  long long* trace;  // optional: CTA 0 records clock64() at pipeline hand-offs, [64 blocks][32]
};

// Forward pipeline trace (CTA 0, first 64 key blocks; only in the kTrace
// instantiation).  Slots: 0-5 softmax warp 2 lane 0 (scores ready, scores
// loaded, row max, exponentials with P written to TMEM, O synchronised /
// rescaled, P handed to the MMA warp), 6-11 the same for warp 6 (split rows),
// 12 / 13 MMA issue of S / P V, 14 / 15 TMA issue of K / V.
#define MD_FTRACE(gg, slot)                                                                      \
  do {                                                                                          \
    if (kTrace && blockIdx.x == 0 && (gg) < 64) p.trace[(gg) * 32 + (slot)] = clock64();        \
  } while (0)

__device__ __forceinline__ void decode(const FwdParams& p, int w, int& qt, int& b, int& h) {
  const int bh_count = p.B * p.H;
  qt = p.n_qt - 1 - w / bh_count;
  const int bh = w % bh_count;
  b = bh / p.H;
  h = bh % p.H;
}

__device__ __forceinline__ float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}
__device__ __forceinline__ float lg2(float x) {
  float y;
  asm("lg2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}


// tm: Q/K/V loads ([B, S, 3*H*D], or [B, S, 3H, dr]); to: output stores
// ([B, S, H*D], or [B, S, H, dr]).
template <int D, bool kTrace>
__global__ void __launch_bounds__(FwdCfg<D>::kThreads, FwdCfg<D>::kCtasPerSm)
    fwd_kernel(const __grid_constant__ CUtensorMap tm, const __grid_constant__ CUtensorMap to,
               const __grid_constant__ FwdParams p) {
  using C = FwdCfg<D>;
  constexpr int KST = C::kKvStages;
  constexpr int QB = C::kQBufs;
  constexpr int SB = C::kSBufs;
  constexpr int PB = C::kPBufs;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sQ = smem;
  uint8_t* sK = sQ + QB * C::kTileBytes;
  uint8_t* sV = sK + KST * C::kTileBytes;
  float* sRed = reinterpret_cast<float*>(sV + KST * C::kTileBytes);  // split rows only
  uint64_t* bars = reinterpret_cast<uint64_t*>(sV + KST * C::kTileBytes + C::kRedBytes);
  uint64_t* q_full = bars;           // [2]
  uint64_t* o_staged = bars + 2;     // [2] the item's O is in its Q buffer (softmax warps -> warp 0)
  uint64_t* k_full = bars + 4;       // [4]
  uint64_t* k_empty = bars + 8;      // [4]
  uint64_t* v_full = bars + 12;      // [4]
  uint64_t* v_empty = bars + 16;     // [4]
  uint64_t* s_full = bars + 20;      // [2]
  uint64_t* s_free = bars + 22;      // [2]
  uint64_t* p_full = bars + 24;
  uint64_t* o_done = bars + 25;
  uint64_t* drain = bars + 26;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 27);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(bars + 28);
  uint64_t* xbar = bars + 29;        // [4] row exchange between the two warps of a lane quarter (split rows)

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int i = 0; i < QB; ++i) {
      mbar_init(&q_full[i], 1);
      mbar_init(&o_staged[i], C::kSoftWarps);
    }
    for (int i = 0; i < KST; ++i) {
      mbar_init(&k_full[i], 1);
      mbar_init(&k_empty[i], 1);
      mbar_init(&v_full[i], 1);
      mbar_init(&v_empty[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&s_full[i], 1);
      mbar_init(&s_free[i], C::kSoftWarps);
    }
    mbar_init(p_full, C::kSoftWarps);
    if (C::kSplit == 2)
      for (int i = 0; i < 4; ++i) mbar_init(&xbar[i], 2);
    mbar_init(o_done, 1);
    mbar_init(drain, 1);
    *abort_flag = 0;
    fence_mbar_init();
    tma_prefetch_desc(&tm);
    tma_prefetch_desc(&to);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, C::kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  // Prologue done: the next kernel may launch; global memory only after the previous one finished.
  pdl_trigger();
  pdl_wait();

  const bool map4 = p.dr != D;  // uniform
  if (warp == 0 && lane == 0) {
    // ------------------------------------------------------------ TMA loads and output stores
    int q_armed[2] = {-1, -1};
    int k_armed[4] = {-1, -1, -1, -1};
    int v_armed[4] = {-1, -1, -1, -1};
    // Store item ti's output tile (staged by the softmax warps in Q buffer ti % QB).
    auto store_out = [&](int ti) -> bool {
      const int qb = ti % QB;
      if (!mbar_wait(&o_staged[qb], static_cast<uint32_t>(ti / QB) & 1u, p.status, 46, abort_flag)) return false;
      int qt, b, h;
      decode(p, blockIdx.x + ti * gridDim.x, qt, b, h);
#pragma unroll
      for (int c = 0; c < C::kChunks; ++c) {
        if (c * 64 >= p.dr) break;  // uniform: nothing of this box lies inside the tensor
        const uint8_t* src = sQ + qb * C::kTileBytes + c * (kBM * 128);
        if (map4) tma_store_4d(&to, src, c * 64, h, qt * kBM, b);
        else tma_store_3d(&to, src, h * D + c * 64, qt * kBM, b);
      }
      bulk_commit_group();
      return true;
    };
    int g = 0, t = 0, stored = 0;
    bool ok = true;
    for (int w = blockIdx.x; w < p.items && ok; w += gridDim.x, ++t) {
      int qt, b, h;
      decode(p, w, qt, b, h);
      const int qb = t % QB;
      if (t >= QB) {
        // Buffer qb last held item t-QB: store that item's output, and reload the
        // buffer once the store has read it.
        if (!store_out(t - QB)) {
          ok = false;
          break;
        }
        stored = t - QB + 1;
        bulk_wait_read_all();
      }
      mbar_arrive_expect_tx(&q_full[qb], C::kTileBytes);
      q_armed[qb] = static_cast<int>(static_cast<uint32_t>(t / QB) & 1u);
      const int col0 = h * 3 * D;
#pragma unroll
      for (int c = 0; c < C::kChunks; ++c) {
        if (map4) tma_load_4d(&tm, &q_full[qb], sQ + qb * C::kTileBytes + c * (kBM * 128), c * 64, 3 * h, qt * kBM, b);
        else tma_load_3d(&tm, &q_full[qb], sQ + qb * C::kTileBytes + c * (kBM * 128), col0 + c * 64, qt * kBM, b);
      }
      for (int j = 0; j <= qt; ++j, ++g) {
        const int st = g % KST;
        const uint32_t ph = static_cast<uint32_t>(g / KST) & 1u;
        if (!mbar_wait(&k_empty[st], ph ^ 1u, p.status, 41, abort_flag)) {
          ok = false;
          break;
        }
        mbar_arrive_expect_tx(&k_full[st], C::kTileBytes);
        k_armed[st] = static_cast<int>(ph);
        MD_FTRACE(g, 14);
#pragma unroll
        for (int c = 0; c < C::kChunks; ++c) {
          if (map4) tma_load_4d(&tm, &k_full[st], sK + st * C::kTileBytes + c * (kBN * 128), c * 64, 3 * h + 1, j * kBN, b);
          else tma_load_3d(&tm, &k_full[st], sK + st * C::kTileBytes + c * (kBN * 128), col0 + D + c * 64, j * kBN, b);
        }
        if (!mbar_wait(&v_empty[st], ph ^ 1u, p.status, 42, abort_flag)) {
          ok = false;
          break;
        }
        mbar_arrive_expect_tx(&v_full[st], C::kTileBytes);
        v_armed[st] = static_cast<int>(ph);
        MD_FTRACE(g, 15);
#pragma unroll
        for (int c = 0; c < C::kChunks; ++c) {
          if (map4) tma_load_4d(&tm, &v_full[st], sV + st * C::kTileBytes + c * (kBN * 128), c * 64, 3 * h + 2, j * kBN, b);
          else tma_load_3d(&tm, &v_full[st], sV + st * C::kTileBytes + c * (kBN * 128), col0 + 2 * D + c * 64,
                           j * kBN, b);
        }
      }
    }
    // The last items' outputs (skipped after an abort: their tiles were never staged).
    if (ok)
      for (int ti = stored; ti < t; ++ti)
        if (!store_out(ti)) break;
    // No bulk copy may still be in flight at exit: stores complete, loads landed.
    bulk_wait_all();
    for (int i = 0; i < QB; ++i)
      if (q_armed[i] >= 0) mbar_wait(&q_full[i], static_cast<uint32_t>(q_armed[i]), p.status, 43, nullptr);
    for (int i = 0; i < KST; ++i) {
      if (k_armed[i] >= 0) mbar_wait(&k_full[i], static_cast<uint32_t>(k_armed[i]), p.status, 44, nullptr);
      if (v_armed[i] >= 0) mbar_wait(&v_full[i], static_cast<uint32_t>(v_armed[i]), p.status, 45, nullptr);
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer (whole warp, elected lane issues)
    constexpr uint32_t idS = idesc_bf16_f32(kBM, kBN, false, false);
    constexpr uint32_t idO = idesc_bf16_f32(kBM, D, false, true);
    // Base descriptors; an operand at byte offset `off` is base + (off >> 4).
    const uint64_t dV = sdesc_sw128(smem_u32(sV), kBN * 128, 1024);
    const uint64_t dQ = sdesc_sw128(smem_u32(sQ), 16, 1024);
    const uint64_t dK = sdesc_sw128(smem_u32(sK), 16, 1024);
    constexpr uint32_t kTile16 = C::kTileBytes >> 4;
    int pend = -1;
    bool pend_first = false;
    // O += P V for block gp (P from TMEM, V MN-major from shared memory).
    auto issue_pv = [&](int gp, bool first) -> bool {
      if (!mbar_wait(p_full, static_cast<uint32_t>(gp) & 1u, p.status, 52, abort_flag)) return false;
      const int st = gp % KST;
      if (!mbar_wait(&v_full[st], static_cast<uint32_t>(gp / KST) & 1u, p.status, 53, abort_flag)) return false;
      tc_fence_after();
      if (lane == 0) MD_FTRACE(gp, 13);
      const uint64_t v0 = dV + st * kTile16;
#pragma unroll
      for (int kk = 0; kk < kBN / 16; ++kk)
        umma_bf16_ts_elect(tmem + C::kOCol, tmem + C::kPCol + static_cast<uint32_t>((gp % C::kPBufs) * (kBN / 2) + kk * 8),
                           v0 + kk * 128, idO, (first && kk == 0) ? 0u : 1u);
      umma_commit_elect(o_done);
      umma_commit_elect(&v_empty[st]);
      return true;
    };
    // While a P V product is pending, issue whichever comes first: that product (its P
    // is in TMEM) or the next score product (its K tile and score buffer are free).
    // Returns 1 when the P V went first, 0 when the scores may go first, -1 on
    // timeout / abort.
    auto pv_first = [&](uint64_t* a, uint32_t pa, uint64_t* b2, uint32_t pb) -> int {
      const uint64_t t0 = globaltimer_ns();
      for (uint32_t it = 0;; ++it) {
        if (mbar_test_wait(a, pa) && (b2 == nullptr || mbar_test_wait(b2, pb))) return 0;
        if (mbar_test_wait(p_full, static_cast<uint32_t>(pend) & 1u)) return issue_pv(pend, pend_first) ? 1 : -1;
        if ((it & 63u) == 63u) {
          if (*abort_flag) return -1;
          if (globaltimer_ns() - t0 > kPipelineTimeoutNs) {
            report(p.status, kTimeoutPipeline, 56, 0);
            *abort_flag = 1;
            return -1;
          }
        }
      }
    };
    int g = 0, t = 0;
    bool ok = true;
    for (int w = blockIdx.x; w < p.items && ok; w += gridDim.x, ++t) {
      int qt, b, h;
      decode(p, w, qt, b, h);
      const int qb = t % QB;
      const uint32_t qph = static_cast<uint32_t>(t / QB) & 1u;
      if (pend >= 0) {
        const int r = pv_first(&q_full[qb], qph, nullptr, 0);
        if (r < 0) {
          ok = false;
          break;
        }
        if (r == 1) pend = -1;
      }
      if (!mbar_wait(&q_full[qb], qph, p.status, 50, abort_flag)) {
        ok = false;
        break;
      }
      const uint64_t q0 = dQ + qb * kTile16;
      for (int j = 0; j <= qt; ++j, ++g) {
        const int st = g % KST;
        const int sb = g % SB;
        const uint32_t kph = static_cast<uint32_t>(g / KST) & 1u;
        const uint32_t sph = (static_cast<uint32_t>(g / SB) & 1u) ^ 1u;
        if (pend >= 0) {
          const int r = pv_first(&k_full[st], kph, &s_free[sb], sph);
          if (r < 0) {
            ok = false;
            break;
          }
          if (r == 1) pend = -1;
        }
        if (!mbar_wait(&k_full[st], kph, p.status, 51, abort_flag) ||
            !mbar_wait(&s_free[sb], sph, p.status, 54, abort_flag)) {
          ok = false;
          break;
        }
        tc_fence_after();
        if (lane == 0) MD_FTRACE(g, 12);
        const uint64_t k0 = dK + st * kTile16;
        const uint32_t sd = tmem + static_cast<uint32_t>(sb * kBN);
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) {
          const uint32_t off = ((kk >> 2) * (kBM * 128) + (kk & 3) * 32) >> 4;
          umma_bf16_ss_elect(sd, q0 + off, k0 + off, idS, kk > 0 ? 1u : 0u);
        }
        umma_commit_elect(&s_full[sb]);
        umma_commit_elect(&k_empty[st]);
        if (pend >= 0 && !issue_pv(pend, pend_first)) {
          ok = false;
          break;
        }
        pend = g;
        pend_first = (j == 0);
      }
    }
    if (ok && pend >= 0) issue_pv(pend, pend_first);
    // Every MMA this warp issued completes before TMEM is released.
    umma_commit_elect(drain);
    mbar_wait(drain, 0, p.status, 55, nullptr);
  } else if (warp >= 2) {
    // ------------------------------------------------------------ softmax + epilogue
    constexpr int NC = kBN / C::kSplit;      // key columns per thread
    constexpr int OC = D / 32 / C::kSplit;   // 32-column O chunks per thread (rescale, epilogue)
    const int half = (warp - 2) >> 2;        // column half of the row (0 unless split)
    const int quarter = warp & 3;
    const int row = quarter * 32 + lane;
    const uint32_t lane_base = static_cast<uint32_t>(quarter * 32) << 16;
    const int kc0 = half * NC;               // first key column of this thread
    const float sl2 = p.scale_log2;
    const int tslot = lane == 0 && quarter == 2 ? 6 * half : -1;  // warps 2 and 6 record (kTrace)
    uint32_t xph = 0;                        // row exchanges done (split rows)
    // Split rows: post(v) publishes v for the partner warp (other column half, same
    // rows); get() returns the partner's value of the same exchange.  Exchange k uses
    // buffer k & 1: a warp rewrites a buffer only after the partner arrived at the
    // next exchange, i.e. after it read this one.  Bounded wait; false on timeout /
    // abort.
    auto post = [&](float v) {
      sRed[(static_cast<int>(xph & 1u) * 2 + half) * kBM + row] = v;
      __syncwarp();
      if (lane == 0) mbar_arrive(&xbar[quarter]);
    };
    auto get = [&](float& v, int site) -> bool {
      if (!mbar_wait(&xbar[quarter], xph & 1u, p.status, site, abort_flag)) return false;
      v = sRed[(static_cast<int>(xph & 1u) * 2 + (half ^ 1)) * kBM + row];
      ++xph;
      return true;
    };
    int g = 0, t = 0;
    for (int w = blockIdx.x; w < p.items; w += gridDim.x, ++t) {
      int qt, b, h;
      decode(p, w, qt, b, h);
      float m = -INFINITY, l = 0.f;  // split rows: l is this half's partial sum
      bool ok = true;
      for (int j = 0; j <= qt; ++j, ++g) {
        const int sb = g % SB;
        if (!mbar_wait(&s_full[sb], static_cast<uint32_t>(g / SB) & 1u, p.status, 60, abort_flag)) {
          ok = false;
          break;
        }
        tc_fence_after();
        if (kTrace && tslot >= 0) MD_FTRACE(g, tslot + 0);
        uint32_t r[NC / 32][32];
#pragma unroll
        for (int c = 0; c < NC / 32; ++c)
          tmem_ld_32x32b_x32(tmem + lane_base + static_cast<uint32_t>(sb * kBN + kc0 + c * 32), r[c]);
        tmem_ld_wait();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&s_free[sb]);
        if (kTrace && tslot >= 0) MD_FTRACE(g, tslot + 1);
        if (j == qt) {  // diagonal block: key > query is masked
#pragma unroll
          for (int c = 0; c < NC / 32; ++c)
#pragma unroll
            for (int i = 0; i < 32; ++i)
              if (kc0 + c * 32 + i > row) r[c][i] = __float_as_uint(-INFINITY);
        }
        // Row maximum over eight independent partial maxima (a short dependency chain).
        float mx8[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) mx8[i] = -INFINITY;
#pragma unroll
        for (int c = 0; c < NC / 32; ++c)
#pragma unroll
          for (int i = 0; i < 32; ++i) mx8[i & 7] = fmaxf(mx8[i & 7], __uint_as_float(r[c][i]));
        float mx = fmaxf(fmaxf(fmaxf(mx8[0], mx8[1]), fmaxf(mx8[2], mx8[3])),
                         fmaxf(fmaxf(mx8[4], mx8[5]), fmaxf(mx8[6], mx8[7])));
        mx *= sl2;
        // Row maximum across a split row: each half posts its own.  Usually neither half
        // moves the (stale) running max, so the exponentials start at once with m and the
        // partner's maximum is read afterwards; in the rare block where it does move the
        // max the halves agree first (or the exponentials are redone).  Both halves apply
        // the same rule to the same values, so they use the same m_use.
        float m_use = m;
        bool agreed = true;
        if constexpr (C::kSplit == 2) {
          post(mx);
          if (__any_sync(0xFFFFFFFFu, mx > m + kRescaleLog2)) {
            float other;
            if (!get(other, 63)) {
              ok = false;
              break;
            }
            mx = fmaxf(mx, other);
          } else {
            agreed = false;
          }
        }
        if (agreed) m_use = mx > m + kRescaleLog2 ? mx : m;
        if (kTrace && tslot >= 0) MD_FTRACE(g, tslot + 2);
        // P V of the previous block must have finished before O is rescaled and, with one
        // P buffer, before this block's P overwrites the one it reads.
        auto wait_pv = [&]() -> bool {
          if (!mbar_wait(o_done, static_cast<uint32_t>(g - 1) & 1u, p.status, 61, abort_flag)) return false;
          tc_fence_after();
          return true;
        };
        if (PB == 1 && j > 0 && !wait_pv()) {
          ok = false;
          break;
        }
        // Exponentials, 64 keys at a time; their bf16 pairs go to TMEM (P buffer g % PB,
        // the A operand of the P V product) as soon as a 32-column group is complete.
        const uint32_t pcol = tmem + lane_base + C::kPCol + static_cast<uint32_t>((g % PB) * (kBN / 2) + half * (NC / 2));
        float l0, l1;
        auto exps = [&](float mu) {
          l0 = 0.f;
          l1 = 0.f;
#pragma unroll
          for (int k = 0; k < NC / 64; ++k) {
            uint32_t pq[32];
#pragma unroll
            for (int cc = 0; cc < 2; ++cc)
#pragma unroll
              for (int i = 0; i < 32; i += 2) {
                const float e0 = ex2(fmaf(__uint_as_float(r[2 * k + cc][i]), sl2, -mu));
                const float e1 = ex2(fmaf(__uint_as_float(r[2 * k + cc][i + 1]), sl2, -mu));
                l0 += e0;
                l1 += e1;
                pq[(cc * 32 + i) >> 1] = pack_bf16x2(e0, e1);
              }
            tmem_st_32x32b_x32(pcol + static_cast<uint32_t>(k * 32), pq);
          }
        };
        exps(m_use);
        if constexpr (C::kSplit == 2) {
          if (!agreed) {
            float other;
            if (!get(other, 63)) {
              ok = false;
              break;
            }
            if (__any_sync(0xFFFFFFFFu, other > m + kRescaleLog2)) {
              // The partner's half moved the max: redo this block's exponentials with it.
              mx = fmaxf(mx, other);
              m_use = mx > m + kRescaleLog2 ? mx : m;
              tmem_st_wait();  // the P columns are rewritten below
              exps(m_use);
            }
          }
        }
        const float alpha = ex2(m - m_use);
        l = l * alpha + (l0 + l1);
        if (kTrace && tslot >= 0) MD_FTRACE(g, tslot + 3);
        if (j > 0) {
          if (PB == 2 && !wait_pv()) {
            ok = false;
            break;
          }
          // Rows of the partner warp make the same decision, so each half rescales its O columns.
          if (__any_sync(0xFFFFFFFFu, m_use != m)) {
#pragma unroll
            for (int c = 0; c < OC; ++c) {
              uint32_t o[32];
              const uint32_t ta = tmem + lane_base + C::kOCol + static_cast<uint32_t>((half * OC + c) * 32);
              tmem_ld_32x32b_x32(ta, o);
              tmem_ld_wait();
#pragma unroll
              for (int i = 0; i < 32; ++i) o[i] = __float_as_uint(__uint_as_float(o[i]) * alpha);
              tmem_st_32x32b_x32(ta, o);
            }
          }
        }
        m = m_use;
        if (kTrace && tslot >= 0) MD_FTRACE(g, tslot + 4);
        tmem_st_wait();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(p_full);
        if (kTrace && tslot >= 0) MD_FTRACE(g, tslot + 5);
      }
      if (!ok) break;
      if constexpr (C::kSplit == 2) {
        float other;
        post(l);
        if (!get(other, 64)) break;
        l += other;
      }
      // Epilogue: O / l from TMEM into the 128B-swizzled staging tile (this item's Q
      // buffer: every score product of the item has completed), lse to global memory.
      if (!mbar_wait(o_done, static_cast<uint32_t>(g - 1) & 1u, p.status, 62, abort_flag)) break;
      tc_fence_after();
      const int q = qt * kBM + row;
      const float inv_l = 1.0f / l;
      uint8_t* stage = sQ + (t % QB) * C::kTileBytes;
#pragma unroll
      for (int cc = 0; cc < OC; ++cc) {
        const int c = half * OC + cc;  // 32-column chunk: atom c / 2, 16-byte groups (c % 2) * 4 + k
        uint32_t o[32];
        tmem_ld_32x32b_x32(tmem + lane_base + C::kOCol + static_cast<uint32_t>(c * 32), o);
        tmem_ld_wait();
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          uint8_t* dst = stage + (c >> 1) * (kBM * 128) + sw128_off(row, (c & 1) * 4 + k);
          asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(smem_u32(dst)),
                       "r"(pack_bf16x2(__uint_as_float(o[8 * k + 0]) * inv_l, __uint_as_float(o[8 * k + 1]) * inv_l)),
                       "r"(pack_bf16x2(__uint_as_float(o[8 * k + 2]) * inv_l, __uint_as_float(o[8 * k + 3]) * inv_l)),
                       "r"(pack_bf16x2(__uint_as_float(o[8 * k + 4]) * inv_l, __uint_as_float(o[8 * k + 5]) * inv_l)),
                       "r"(pack_bf16x2(__uint_as_float(o[8 * k + 6]) * inv_l, __uint_as_float(o[8 * k + 7]) * inv_l))
                       : "memory");
        }
      }
      if (half == 0 && q < p.S)
        p.lse[(static_cast<long long>(b) * p.H + h) * p.S + q] = (m + lg2(l)) * 0.6931471805599453f;
      fence_proxy_async_smem();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&o_staged[t % QB]);
    }
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) tmem_dealloc(tmem, C::kTmemCols);
}

#undef MD_FTRACE



// ===========================================================================
// Backward
//
// One work item = (key tile kt of 128 keys, batch*head); items ordered
// longest-first (tile kt meets nqt - kt query blocks).  Per query block i:
//   S^T  = K Q_i^T          (TMEM, 128 keys x 128 queries)
//   dP^T = V dO_i^T         (TMEM)
//   P^T  = exp(S^T * scale - lse_i),  dS^T = P^T (dP^T - delta_i)   [compute warps, bf16:
//                                             P^T to TMEM, dS^T to shared memory]
//   dV  += P^T dO_i,   dK += dS^T Q_i      (TMEM accumulators for the whole item; dV reads
//                                             P^T from TMEM as its A operand)
//   dQ_i = dS K_j                            (TMEM, drained by the dQ warps into an
//                                             fp32 accumulator with bulk reduce-adds)
// Roles: warp 0 TMA, warp 1 MMA, warps 2..9 compute (thread = key row; warps
// 2..5 take query columns 0..63, warps 6..9 columns 64..127, so two warps
// share every SM sub-partition), warps 10..13 dQ drain (thread = query row,
// staged through shared memory into bulk reduce-adds).
// The tensor core runs the next block's score products as soon as the compute
// warps hold this block's scores in registers and its Q/dO tile has landed (or,
// when this block's P^T/dS^T are ready first, right after this block's
// products), then dK and dQ (which read dS^T; a single buffer, released as
// soon as they are done), then dV (which reads P^T; the compute warps write the
// next block's P^T once it has finished).  Q/dO tiles stream through three
// stages.  K/V are double-buffered: the next item's tiles load while this item
// runs, and a finished item's dK / dV are staged (bf16, 128B-swizzled) in its
// own K / V buffers and written by the TMA warp with bulk tensor stores, after
// which the buffers are reloaded -- so an item boundary costs neither a K/V
// load nor the compute warps' time for scattered global stores.
// ===========================================================================
constexpr int kBwdThreads = 448;
constexpr int kBwdCompute = 8;  // compute warps

template <int D>
struct BwdCfg {
  static constexpr int kChunks = D / 64;
  static constexpr int kTileBytes = 128 * D * 2;
  static constexpr int kQStages = 3;
  static constexpr int kPBytes = 128 * 128 * 2;       // dS^T (bf16)
  static constexpr int kStgBytes = 128 * D * 4;       // dQ staging (fp32, D / 32 boxes [128][32])
  // (K, V) x 2 | (Q, dO) x stages | dS^T | dQ staging | lse, delta x 2 blocks
  static constexpr int kSmemData = (4 + 2 * kQStages) * kTileBytes + kPBytes + kStgBytes + 2 * 2 * 128 * 4;
  // No alignment slack fits: the dynamic window must start 1024-byte aligned
  // (checked in the kernel).
  static constexpr int kSmemBytes = kSmemData + 256;
  static constexpr uint32_t kTmemCols = 512;
  // P^T (bf16 pairs, 64 columns) is the A operand of dV += P^T dO.
  static constexpr uint32_t kColS = 0, kColDP = 128, kColDV = 256, kColDK = 256 + D, kColDQ = 256 + 2 * D,
                            kColP = 256 + 3 * D;
  static_assert(256 + 3 * D + 64 <= 512, "TMEM budget");
  static_assert(kSmemBytes <= 232448, "shared memory budget");
};

struct BwdParams {
  const float* lse;    // [B, H, S] natural log
  const float* delta;  // [B, H, S]
  float* dqacc;        // [B*S, ldacc] fp32, zeroed
  long long ldacc;
  void* dqkv;          // [B*S, lddq] bf16 interleaved [H, 3, D]
  long long lddq;
  int B, H, S;
  int n_t;             // 128-row tiles per sequence
  int items;
  float scale, scale_log2;
  int flags;           // bit 0: skip the dQ reductions (timing experiments only; dQ is then wrong)
  Status* status;
  long long* trace;    // optional: CTA 0 records clock64() at pipeline hand-offs, [64 blocks][32]
};

// Pipeline trace for performance analysis (CTA 0, first 64 blocks; only in the
// kTrace instantiation).
#define MD_TRACE(gg, slot)                                                                  \
  do {                                                                                     \
    if (kTrace && blockIdx.x == 0 && (gg) < 64) p.trace[(gg) * 32 + (slot)] = clock64();   \
  } while (0)


template <int D, bool kTrace>
__global__ void __launch_bounds__(kBwdThreads, 1)
    bwd_kernel(const __grid_constant__ CUtensorMap tmQKV, const __grid_constant__ CUtensorMap tmDO,
               const __grid_constant__ CUtensorMap tmDQ, const __grid_constant__ CUtensorMap tmOut,
               const __grid_constant__ BwdParams p) {
  using C = BwdCfg<D>;
  constexpr int QS = C::kQStages;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  if ((smem_u32(smem_raw) & 1023u) != 0u) {  // uniform across the CTA
    if (threadIdx.x == 0) report(p.status, kBadArgument, 69, smem_u32(smem_raw));
    return;
  }
  uint8_t* sKV = smem_raw;                        // [2] x (K, V); K of buffer kb at sKV + 2 kb tile
  uint8_t* sQ = sKV + 4 * C::kTileBytes;          // [QS]
  uint8_t* sdO = sQ + QS * C::kTileBytes;         // [QS]
  uint8_t* sdSt = sdO + QS * C::kTileBytes;       // dS^T
  uint8_t* sStg = sdSt + C::kPBytes;              // dQ staging
  float* sL = reinterpret_cast<float*>(sStg + C::kStgBytes);  // [2][128] lse (log2 units)
  float* sDel = sL + 2 * 128;                                   // [2][128]
  uint64_t* bars = reinterpret_cast<uint64_t*>(sDel + 2 * 128);
  static_assert(QS == 3, "barrier slots below are laid out for three Q/dO stages");
  uint64_t* kv_full = bars + 0;    // [2]
  uint64_t* qd_full = bars + 2;    // [3]
  uint64_t* qd_empty = bars + 5;   // [3]
  uint64_t* kv_staged = bars + 26; // [2] the item's dK / dV are in its K / V buffers
  uint64_t* sd_full = bars + 8;
  uint64_t* sd_free = bars + 9;
  uint64_t* pds_full = bars + 10;
  uint64_t* p_free = bars + 11;    // [2] by block parity: dV of the block has completed
  uint64_t* ds_free = bars + 13;
  uint64_t* dq_full = bars + 14;
  uint64_t* dq_free = bars + 15;
  uint64_t* dkv_free = bars + 16;
  uint64_t* drain = bars + 17;
  uint64_t* stage_bar = bars + 18;  // [2] (slot 20 unused)
  uint64_t* pst_free = bars + 21;   // [0]: the dQ staging tile has been read by the reduce-adds (slot 22 unused)
  uint64_t* dq_staged = bars + 23;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 24);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(bars + 25);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int bhc = p.B * p.H;

  if (threadIdx.x == 0) {
    for (int i = 0; i < 2; ++i) {
      mbar_init(&kv_full[i], 1);
      mbar_init(&kv_staged[i], kBwdCompute);
    }
    for (int i = 0; i < QS; ++i) {
      mbar_init(&qd_full[i], 1);
      mbar_init(&qd_empty[i], 1);
    }
    mbar_init(sd_full, 1);
    mbar_init(sd_free, kBwdCompute);
    mbar_init(pds_full, kBwdCompute);
    mbar_init(&p_free[0], 1);
    mbar_init(&p_free[1], 1);
    mbar_init(ds_free, 1);
    mbar_init(dq_full, 1);
    mbar_init(dq_free, 4);
    mbar_init(dkv_free, kBwdCompute);
    mbar_init(drain, 1);
    for (int i = 0; i < 2; ++i) mbar_init(&stage_bar[i], kBwdCompute);
    mbar_init(&pst_free[0], 1);
    mbar_init(&pst_free[1], 1);
    mbar_init(dq_staged, 4);
    *abort_flag = 0;
    fence_mbar_init();
    tma_prefetch_desc(&tmQKV);
    tma_prefetch_desc(&tmDO);
    tma_prefetch_desc(&tmDQ);
    tma_prefetch_desc(&tmOut);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, C::kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  // Prologue done: the next kernel may launch; global memory only after the previous one finished.
  pdl_trigger();
  pdl_wait();

  if (warp == 0 && lane == 0) {
    // ------------------------------------------------------------ TMA loads and dK / dV stores
    int kv_armed[2] = {-1, -1};
    int q_armed[QS];
    for (int i = 0; i < QS; ++i) q_armed[i] = -1;
    // Store item ti's dK / dV (staged by the compute warps in K / V buffer ti % 2).
    auto store_dkv = [&](int ti) -> bool {
      const int kb = ti & 1;
      if (!mbar_wait(&kv_staged[kb], static_cast<uint32_t>(ti >> 1) & 1u, p.status, 74, abort_flag)) return false;
      const int w = blockIdx.x + ti * gridDim.x;
      const int kt = w / bhc, bh = w % bhc, b = bh / p.H, h = bh % p.H;
      const uint8_t* sk = sKV + 2 * kb * C::kTileBytes;
#pragma unroll
      for (int c = 0; c < C::kChunks; ++c) {
        tma_store_3d(&tmOut, sk + c * 16384, h * 3 * D + D + c * 64, kt * 128, b);
        tma_store_3d(&tmOut, sk + C::kTileBytes + c * 16384, h * 3 * D + 2 * D + c * 64, kt * 128, b);
      }
      bulk_commit_group();
      return true;
    };
    int g = 0, t = 0, stored = 0;
    bool ok = true;
    for (int w = blockIdx.x; w < p.items && ok; w += gridDim.x, ++t) {
      const int kt = w / bhc, bh = w % bhc, b = bh / p.H, h = bh % p.H;
      const int kb = t & 1;
      if (t >= 2) {
        // Buffer kb last held item t-2: store its dK / dV, reload once the store has read them.
        if (!store_dkv(t - 2)) {
          ok = false;
          break;
        }
        stored = t - 1;
        bulk_wait_read_all();
      }
      mbar_arrive_expect_tx(&kv_full[kb], 2 * C::kTileBytes);
      kv_armed[kb] = static_cast<int>(static_cast<uint32_t>(t >> 1) & 1u);
      const int col0 = h * 3 * D;
      uint8_t* sk = sKV + 2 * kb * C::kTileBytes;
#pragma unroll
      for (int c = 0; c < C::kChunks; ++c) {
        tma_load_3d(&tmQKV, &kv_full[kb], sk + c * 16384, col0 + D + c * 64, kt * 128, b);
        tma_load_3d(&tmQKV, &kv_full[kb], sk + C::kTileBytes + c * 16384, col0 + 2 * D + c * 64, kt * 128, b);
      }
      for (int i = kt; i < p.n_t; ++i, ++g) {
        const int st = g % QS;
        const uint32_t ph = static_cast<uint32_t>(g / QS) & 1u;
        if (!mbar_wait(&qd_empty[st], ph ^ 1u, p.status, 71, abort_flag)) {
          ok = false;
          break;
        }
        MD_TRACE(g, 11);
        mbar_arrive_expect_tx(&qd_full[st], 2 * C::kTileBytes);
        q_armed[st] = static_cast<int>(ph);
#pragma unroll
        for (int c = 0; c < C::kChunks; ++c) {
          tma_load_3d(&tmQKV, &qd_full[st], sQ + st * C::kTileBytes + c * 16384, col0 + c * 64, i * 128, b);
          tma_load_3d(&tmDO, &qd_full[st], sdO + st * C::kTileBytes + c * 16384, h * D + c * 64, i * 128, b);
        }
      }
    }
    // The last items' dK / dV (skipped after an abort: they were never staged).
    if (ok)
      for (int ti = stored; ti < t; ++ti)
        if (!store_dkv(ti)) break;
    bulk_wait_all();
    for (int i = 0; i < 2; ++i)
      if (kv_armed[i] >= 0) mbar_wait(&kv_full[i], static_cast<uint32_t>(kv_armed[i]), p.status, 72, nullptr);
    for (int i = 0; i < QS; ++i)
      if (q_armed[i] >= 0) mbar_wait(&qd_full[i], static_cast<uint32_t>(q_armed[i]), p.status, 73, nullptr);
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer (whole warp, elected lane issues)
    constexpr uint32_t idS = idesc_bf16_f32(128, 128, false, false);   // S^T, dP^T
    constexpr uint32_t idKV = idesc_bf16_f32(128, D, false, true);     // dV, dK: B MN-major
    constexpr uint32_t idQ = idesc_bf16_f32(128, D, true, true);       // dQ: A (dS) and B (K) MN-major
    // Base descriptors; an operand at byte offset `off` is base + (off >> 4).
    // K / V buffer kb: + 2 kb (K) or 2 kb + 1 (V) tiles.
    const uint64_t dK_k0 = sdesc_sw128(smem_u32(sKV), 16, 1024);
    const uint64_t dK_mn0 = sdesc_sw128(smem_u32(sKV), 16384, 1024);
    const uint64_t dV_k0 = sdesc_sw128(smem_u32(sKV + C::kTileBytes), 16, 1024);
    const uint64_t dQ_k = sdesc_sw128(smem_u32(sQ), 16, 1024);
    const uint64_t dQ_mn = sdesc_sw128(smem_u32(sQ), 16384, 1024);
    const uint64_t ddO_k = sdesc_sw128(smem_u32(sdO), 16, 1024);
    const uint64_t ddO_mn = sdesc_sw128(smem_u32(sdO), 16384, 1024);
    const uint64_t ddS_k = sdesc_sw128(smem_u32(sdSt), 16, 1024);
    const uint64_t ddS_mn = sdesc_sw128(smem_u32(sdSt), 16384, 1024);
    constexpr uint32_t kTile16 = C::kTileBytes >> 4;
    int g = 0, t = 0;
    bool ok = true;
    uint64_t dK_k = dK_k0, dK_mn = dK_mn0, dV_k = dV_k0;  // this item's K / V buffer
    // Score products for block gg.
    auto issue_scores = [&](int gg) -> bool {
      const int st = gg % QS;
      if (!mbar_wait(&qd_full[st], static_cast<uint32_t>(gg / QS) & 1u, p.status, 80, abort_flag) ||
          !mbar_wait(sd_free, (static_cast<uint32_t>(gg) & 1u) ^ 1u, p.status, 81, abort_flag))
        return false;
      MD_TRACE(gg, 12);
      tc_fence_after();
      const uint64_t q0 = dQ_k + st * kTile16, o0 = ddO_k + st * kTile16;
#pragma unroll
      for (int kk = 0; kk < D / 16; ++kk) {
        const uint32_t off = ((kk >> 2) * 16384 + (kk & 3) * 32) >> 4;
        umma_bf16_ss_elect(tmem + C::kColS, dK_k + off, q0 + off, idS, kk > 0 ? 1u : 0u);
        umma_bf16_ss_elect(tmem + C::kColDP, dV_k + off, o0 + off, idS, kk > 0 ? 1u : 0u);
      }
      umma_commit_elect(sd_full);
      return true;
    };
    for (int w = blockIdx.x; w < p.items && ok; w += gridDim.x, ++t) {
      const int kt = w / bhc;
      const int n = p.n_t - kt;
      const int kb = t & 1;
      if (!mbar_wait(&kv_full[kb], static_cast<uint32_t>(t >> 1) & 1u, p.status, 82, abort_flag)) break;
      dK_k = dK_k0 + 2 * kb * kTile16;
      dK_mn = dK_mn0 + 2 * kb * kTile16;
      dV_k = dV_k0 + 2 * kb * kTile16;
      if (!issue_scores(g)) break;
      for (int u = 0; u < n; ++u, ++g) {
        const int st = g % QS;
        const int pb = g & 1;
        // The next block's score products normally go first: they only need the compute
        // warps to have read this block's scores into registers (mid-block) and the next
        // Q / dO tile, so they run while the compute warps finish this block.  If this
        // block's P / dS arrive before that tile has landed, its products go first.
        bool scores_after = false;
        if (u + 1 < n) {
          const int st1 = (g + 1) % QS;
          const uint64_t t0 = globaltimer_ns();
          for (uint32_t it = 0;; ++it) {
            if (mbar_test_wait(&qd_full[st1], static_cast<uint32_t>((g + 1) / QS) & 1u) &&
                mbar_test_wait(sd_free, (static_cast<uint32_t>(g + 1) & 1u) ^ 1u))
              break;
            if (mbar_test_wait(pds_full, static_cast<uint32_t>(g) & 1u)) {
              scores_after = true;
              break;
            }
            if ((it & 63u) == 63u && (*abort_flag || globaltimer_ns() - t0 > kPipelineTimeoutNs)) {
              if (!*abort_flag) {
                report(p.status, kTimeoutPipeline, 87, 0);
                *abort_flag = 1;
              }
              ok = false;
              break;
            }
          }
          if (!ok) break;
          if (!scores_after && !issue_scores(g + 1)) {
            ok = false;
            break;
          }
        }
        MD_TRACE(g, 6);
        if (!mbar_wait(pds_full, static_cast<uint32_t>(g) & 1u, p.status, 83, abort_flag)) {
          ok = false;
          break;
        }
        MD_TRACE(g, 5);
        if (u == 0 && !mbar_wait(dkv_free, (static_cast<uint32_t>(t) & 1u) ^ 1u, p.status, 84, abort_flag)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint64_t qmn = dQ_mn + st * kTile16, omn = ddO_mn + st * kTile16;
        const uint32_t acc0 = u > 0 ? 1u : 0u;
#pragma unroll
        for (int kk = 0; kk < 8; ++kk)
          umma_bf16_ss_elect(tmem + C::kColDK, ddS_k + (((kk >> 2) * 16384 + (kk & 3) * 32) >> 4), qmn + kk * 128,
                             idKV, (acc0 | kk) ? 1u : 0u);
        if (!mbar_wait(dq_free, (static_cast<uint32_t>(g) & 1u) ^ 1u, p.status, 85, abort_flag)) {
          ok = false;
          break;
        }
        MD_TRACE(g, 7);
        tc_fence_after();
#pragma unroll
        for (int kk = 0; kk < 8; ++kk)
          umma_bf16_ss_elect(tmem + C::kColDQ, ddS_mn + kk * 128, dK_mn + kk * 128, idQ, kk > 0 ? 1u : 0u);
        umma_commit_elect(ds_free);
        umma_commit_elect(dq_full);
        // dV += P^T dO with P^T from TMEM (8 columns per 16 queries).
#pragma unroll
        for (int kk = 0; kk < 8; ++kk)
          umma_bf16_ts_elect(tmem + C::kColDV, tmem + C::kColP + static_cast<uint32_t>(kk * 8), omn + kk * 128, idKV,
                             (acc0 | kk) ? 1u : 0u);
        umma_commit_elect(&qd_empty[st]);
        umma_commit_elect(&p_free[pb]);
        MD_TRACE(g, 8);
        if (scores_after && !issue_scores(g + 1)) {
          ok = false;
          break;
        }
      }
      if (!ok) break;
    }
    umma_commit_elect(drain);
    mbar_wait(drain, 0, p.status, 86, nullptr);
  } else if (warp >= 2 && warp < 2 + kBwdCompute) {
    // ------------------------------------------------------------ compute (thread = key row)
    const int quarter = warp & 3;
    const int half = (warp - 2) >> 2;  // query columns [64*half, 64*half + 64)
    const int krow = quarter * 32 + lane;
    const uint32_t lane_base = static_cast<uint32_t>(quarter * 32) << 16;
    const int ct = threadIdx.x - 64;  // 0..255
    // Threads 0..127 stage lse (log2 units), 128..255 delta, one entry per
    // block, one block ahead: block g+1's values go to buffer (g+1) & 1 in the
    // middle of block g, right after the wait for dK/dQ of block g-1 (which
    // implies every compute warp has finished block g-1 and its reads of that
    // buffer); the 8 warps then meet on stage_bar[(g+1) & 1] (bounded wait at
    // the start of block g+1, normally already complete).  The load for block
    // g+2 uses a clamped index and is only scaled when stored, so no
    // arithmetic waits on it meanwhile.
    // The prefetch walks this CTA's blocks with a row pointer per item (one integer
    // division per item, none per block); the value is loaded a block before it is staged.
    const float* const src = ct < 128 ? p.lse : p.delta;
    auto row_of = [&](int w_) -> const float* { return src + static_cast<long long>(w_ % bhc) * p.S; };
    auto load_raw = [&](const float* row, int i_) -> float { return row[min(i_ * 128 + (ct & 127), p.S - 1)]; };
    auto stage = [&](int gg, int i_, float raw) {
      const int q = i_ * 128 + (ct & 127);
      const float v = ct < 128 ? (q < p.S ? raw * 1.4426950408889634f : INFINITY) : (q < p.S ? raw : 0.f);
      (ct < 128 ? sL : sDel)[(gg & 1) * 128 + (ct & 127)] = v;
      __syncwarp();
      if (lane == 0) {
        MD_TRACE(gg, 24 + warp - 2);
        mbar_arrive(&stage_bar[gg & 1]);
      }
    };
    // Advance (w_, i_, row) to the next block of this CTA's work list (w_ = -1 past the end).
    auto next_block = [&](int& w_, int& i_, const float*& row) {
      if (i_ + 1 < p.n_t) {
        ++i_;
      } else if (w_ + static_cast<int>(gridDim.x) < p.items) {
        w_ += static_cast<int>(gridDim.x);
        i_ = w_ / bhc;
        row = row_of(w_);
      } else {
        w_ = -1;
      }
    };
    float pre = 0.f;
    int pre_w = -1, pre_i = 0;  // block whose raw value `pre` holds
    const float* pre_row = src;
    if (static_cast<int>(blockIdx.x) < p.items) {
      pre_w = blockIdx.x;
      pre_i = pre_w / bhc;
      pre_row = row_of(pre_w);
      stage(0, pre_i, load_raw(pre_row, pre_i));
      next_block(pre_w, pre_i, pre_row);
      pre = load_raw(pre_row, pre_i);  // unconditional (a valid row): no select on the loaded value
    }
    int g = 0, t = 0;
    bool ok = true;
    for (int w = blockIdx.x; w < p.items && ok; w += gridDim.x) {
      const int kt = w / bhc;
      const int n = p.n_t - kt;
      for (int u = 0; u < n; ++u, ++g) {
        if (!mbar_wait(&stage_bar[g & 1], static_cast<uint32_t>(g >> 1) & 1u, p.status, 89, abort_flag)) {
          ok = false;
          break;
        }
        if (threadIdx.x == 64) MD_TRACE(g, 0);
        const float* L = sL + (g & 1) * 128 + half * 64;
        const float* Dl = sDel + (g & 1) * 128 + half * 64;
        if (!mbar_wait(sd_full, static_cast<uint32_t>(g) & 1u, p.status, 90, abort_flag)) {
          ok = false;
          break;
        }
        if (threadIdx.x == 64) MD_TRACE(g, 1);
        tc_fence_after();
        uint8_t* sdS = sdSt + half * 16384;
#pragma unroll 1
        for (int c = 0; c < 2; ++c) {
          const uint32_t col = static_cast<uint32_t>(half * 64 + c * 32);
          uint32_t sv[32], dv[32];
          if (c == 1 && threadIdx.x == 64) MD_TRACE(g, 13);
          tmem_ld_32x32b_x32(tmem + lane_base + C::kColS + col, sv);
          tmem_ld_32x32b_x32(tmem + lane_base + C::kColDP + col, dv);
          tmem_ld_wait();
          if (c == 1 && threadIdx.x == 64) MD_TRACE(g, 14);
          if (c == 1) {
            // S^T and dP^T fully read: the next block's score products may overwrite them.
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(sd_free);
          }
          uint32_t pp[16], dd[16];
          float4 l4, d4;  // lse / delta of four queries (one 16-byte broadcast load each)
#pragma unroll
          for (int e = 0; e < 32; e += 2) {
            const int qc = c * 32 + e;  // within this half
            if ((e & 3) == 0) {
              l4 = *reinterpret_cast<const float4*>(L + qc);
              d4 = *reinterpret_cast<const float4*>(Dl + qc);
            }
            const float la = (e & 3) ? l4.z : l4.x, lb = (e & 3) ? l4.w : l4.y;
            const float da = (e & 3) ? d4.z : d4.x, db = (e & 3) ? d4.w : d4.y;
            float p0 = ex2(fmaf(__uint_as_float(sv[e]), p.scale_log2, -la));
            float p1 = ex2(fmaf(__uint_as_float(sv[e + 1]), p.scale_log2, -lb));
            if (u == 0) {  // diagonal block: query < key is masked
              if (half * 64 + qc < krow) p0 = 0.f;
              if (half * 64 + qc + 1 < krow) p1 = 0.f;
            }
            const float g0 = p0 * (__uint_as_float(dv[e]) - da);
            const float g1 = p1 * (__uint_as_float(dv[e + 1]) - db);
            pp[e >> 1] = pack_bf16x2(p0, p1);
            dd[e >> 1] = pack_bf16x2(g0, g1);
          }
          if (c == 1 && threadIdx.x == 64) MD_TRACE(g, 15);
          if (c == 0) {
            if (threadIdx.x == 64) MD_TRACE(g, 2);
            // dV of block g-1 has finished reading P^T (TMEM); dK/dQ of block g-1
            // have finished reading dS^T.
            if ((g >= 1 && !mbar_wait(&p_free[(g - 1) & 1], static_cast<uint32_t>((g - 1) >> 1) & 1u, p.status, 91,
                                      abort_flag)) ||
                (g >= 1 && !mbar_wait(ds_free, static_cast<uint32_t>(g - 1) & 1u, p.status, 93, abort_flag))) {
              ok = false;
              break;
            }
            if (threadIdx.x == 64) MD_TRACE(g, 3);
          }
          // P^T to TMEM (16 columns = these 32 queries), dS^T to shared memory.
          tc_fence_after();
          tmem_st_32x32b_x16(tmem + lane_base + C::kColP + static_cast<uint32_t>(half * 32 + c * 16), pp);
#pragma unroll
          for (int k = 0; k < 4; ++k) {
            const uint32_t off = sw128_off(krow, c * 4 + k);
            asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(smem_u32(sdS + off)), "r"(dd[4 * k]),
                         "r"(dd[4 * k + 1]), "r"(dd[4 * k + 2]), "r"(dd[4 * k + 3])
                         : "memory");
          }
          if (c == 0 && threadIdx.x == 64) MD_TRACE(g, 10);
        }
        if (!ok) break;
        tmem_st_wait();
        fence_proxy_async_smem();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) {
          MD_TRACE(g, 16 + warp - 2);
          mbar_arrive(pds_full);
        }
        // Stage the next block's lse/delta (buffer (g+1) & 1 is free: the wait for dK/dQ
        // of block g-1 above implies every compute warp has finished block g-1), off the
        // path to the P/dS hand-off.
        if (pre_w >= 0) {
          stage(g + 1, pre_i, pre);
          next_block(pre_w, pre_i, pre_row);
          pre = load_raw(pre_row, pre_i);
        }
        if (threadIdx.x == 64) MD_TRACE(g, 4);
      }
      if (!ok) break;
      // dK (scaled; warps of half 0) and dV (half 1) of this key tile, staged as bf16 in
      // the item's K / V buffer (the 128B-swizzled layout the bulk tensor store reads).
      // dV (the last product of the last block) done: both accumulators are final and
      // every product of the item that read K or V has completed.
      if (!mbar_wait(&p_free[(g - 1) & 1], static_cast<uint32_t>((g - 1) >> 1) & 1u, p.status, 92, abort_flag)) break;
      tc_fence_after();
      const float sc = half == 0 ? p.scale : 1.f;
      const uint32_t colx = half == 0 ? C::kColDK : C::kColDV;
      uint8_t* stg = sKV + (2 * (t & 1) + half) * C::kTileBytes;
#pragma unroll
      for (int c = 0; c < D / 32; ++c) {
        uint32_t o[32];
        tmem_ld_32x32b_x32(tmem + lane_base + colx + c * 32, o);
        tmem_ld_wait();
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          uint8_t* dst = stg + (c >> 1) * 16384 + sw128_off(krow, (c & 1) * 4 + k);
          asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(smem_u32(dst)),
                       "r"(pack_bf16x2(__uint_as_float(o[8 * k + 0]) * sc, __uint_as_float(o[8 * k + 1]) * sc)),
                       "r"(pack_bf16x2(__uint_as_float(o[8 * k + 2]) * sc, __uint_as_float(o[8 * k + 3]) * sc)),
                       "r"(pack_bf16x2(__uint_as_float(o[8 * k + 4]) * sc, __uint_as_float(o[8 * k + 5]) * sc)),
                       "r"(pack_bf16x2(__uint_as_float(o[8 * k + 6]) * sc, __uint_as_float(o[8 * k + 7]) * sc))
                       : "memory");
        }
      }
      fence_proxy_async_smem();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) {
        mbar_arrive(dkv_free);
        mbar_arrive(&kv_staged[t & 1]);
      }
      ++t;
    }
  } else if (warp >= 2 + kBwdCompute) {
    // ------------------------------------------------------------ dQ drain (thread = query row)
    // dQ_i leaves TMEM into the staging tile (fp32, two 128 x 32 sub-tiles with
    // the 128-byte swizzle) once the previous block's reduce-adds have read it,
    // then one bulk tensor reduce-add per sub-tile adds it into the fp32
    // accumulator in global memory (the L2 reduces whole lines; rows past the
    // sequence end are clipped by the tensor map).
    const int quarter = warp & 3;
    const int qrow = quarter * 32 + lane;
    const uint32_t lane_base = static_cast<uint32_t>(quarter * 32) << 16;
    const bool issuer = warp == 2 + kBwdCompute && lane == 0;
    int g = 0;
    bool ok = true;
    for (int w = blockIdx.x; w < p.items && ok; w += gridDim.x) {
      const int kt = w / bhc, bh = w % bhc, b = bh / p.H, h = bh % p.H;
      for (int i = kt; i < p.n_t; ++i, ++g) {
        if (!mbar_wait(dq_full, static_cast<uint32_t>(g) & 1u, p.status, 95, abort_flag)) {
          ok = false;
          break;
        }
        if (threadIdx.x == 320) MD_TRACE(g, 9);
        tc_fence_after();
        uint32_t o[D / 32][32];
#pragma unroll
        for (int c = 0; c < D / 32; ++c) tmem_ld_32x32b_x32(tmem + lane_base + C::kColDQ + c * 32, o[c]);
        tmem_ld_wait();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(dq_free);
        // The previous block's reduce-adds have read the staging tile.
        if (g >= 1 && !mbar_wait(&pst_free[0], static_cast<uint32_t>(g - 1) & 1u, p.status, 96, abort_flag)) {
          ok = false;
          break;
        }
        uint8_t* stg = sStg;
#pragma unroll
        for (int c = 0; c < D / 32; ++c)
#pragma unroll
          for (int k = 0; k < 8; ++k)
            asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(smem_u32(stg + c * 16384 +
                                                                                   sw128_off(qrow, k))),
                         "r"(o[c][4 * k]), "r"(o[c][4 * k + 1]), "r"(o[c][4 * k + 2]), "r"(o[c][4 * k + 3])
                         : "memory");
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) mbar_arrive(dq_staged);
        if (issuer) {
          if (!mbar_wait(dq_staged, static_cast<uint32_t>(g) & 1u, p.status, 97, abort_flag)) {
            ok = false;
          } else {
            if (!(p.flags & 1)) {
#pragma unroll
              for (int c = 0; c < D / 32; ++c) tma_reduce_add_3d(&tmDQ, stg + c * 16384, h * D + c * 32, i * 128, b);
              bulk_commit_group();
              bulk_wait_read_all();
            }
            mbar_arrive(&pst_free[0]);
          }
        }
        ok = __shfl_sync(0xFFFFFFFFu, ok ? 1 : 0, 0) != 0;
      }
    }
    if (issuer) bulk_wait_all();
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) tmem_dealloc(tmem, C::kTmemCols);
}


// ===========================================================================
// Backward, head_dim 128 (and 80 on zero-padded boxes)
//
// The head_dim 64 layout needs S^T, dP^T (128 queries each), dK, dV and dQ
// accumulators = 256 + 3 D TMEM columns, 640 at D = 128 (512 exist).  This
// kernel walks each 128-key tile's queries in blocks of 64 and computes dQ
// transposed, dQ^T = K^T dS^T (M = D = 128 rows, N = 64 queries), so
//   S^T 64 | dP^T 64 | dQ^T 64 | P^T 2 x 32 | dK 128 | dV 128  = 512 columns.
// Per 64-query block i of key tile kt:
//   S^T  = K Q_i^T,  dP^T = V dO_i^T                 (M 128 keys, N 64)
//   P^T  = exp(S^T scale - lse_i),  dS^T = P^T (dP^T - delta_i)   [compute warps, bf16:
//                                                     P^T to TMEM, dS^T to shared memory]
//   dK  += dS^T Q_i,  dV += P^T dO_i                 (M 128 keys, N D, K 64; dV reads P^T
//                                                     from TMEM as its A operand)
//   dQ_i^T = K^T dS^T                                (M D, N 64, K 128 keys; both operands MN-major)
// Roles as in the head_dim 64 kernel: warp 0 TMA, warp 1 MMA, warps 2..9
// compute (thread = key row; warps 2..5 take query columns 0..31 of the
// block, 6..9 columns 32..63), warps 10..13 drain dQ^T (thread = head-dim
// row) into a dedicated fp32 staging tile [64 queries][128] (four 128B-
// swizzled boxes of 32 columns) and one bulk tensor reduce-add per box into
// the fp32 accumulator.  Three Q/dO stages, P^T double-buffered in TMEM,
// dS^T single-buffered; the MMA warp queues the next block's score products as
// soon as the compute warps hold the current scores in registers and the next
// Q/dO tile has landed, or after the current block's products when its P/dS
// are ready first.  K/V stay single-buffered (shared memory has no room for a
// second 64 KB pair): an item's dK / dV are staged bf16 in the K / V buffers and
// written by the TMA warp's bulk tensor stores before it reloads them.
// Real head_dim dr <= 128: every tensor map is 4-D [B, S, slots, dr], so
// boxes read zeros past dr and the dQ reduce-add and the dK / dV stores clip
// there.
// ===========================================================================
struct Bwd128Cfg {
  static constexpr int D = 128;
  static constexpr int kBQ = 64;                              // queries per block
  static constexpr int kKTile = 128 * D * 2;                  // K or V tile: 2 chunks [128][64]
  static constexpr int kQTile = kBQ * D * 2;                  // Q or dO tile: 2 chunks [64][64]
  static constexpr int kQChunk = kBQ * 128;                   // 8 KB
  static constexpr int kQStages = 3;
  static constexpr int kPBytes = 128 * kBQ * 2;               // dS^T [128 keys][64 queries]
  static constexpr int kStgBytes = kBQ * D * 4;               // dQ staging, 4 boxes [64][32] fp32
  static constexpr int kSmemData = 2 * kKTile + 2 * kQStages * kQTile + kPBytes + kStgBytes + 2 * 2 * kBQ * 4;
  static constexpr int kSmemBytes = kSmemData + 256;
  static constexpr uint32_t kTmemCols = 512;
  // P^T (bf16 pairs, 32 columns per buffer, two buffers) is the A operand of dV += P^T dO.
  static constexpr uint32_t kColS = 0, kColDP = 64, kColDQ = 128, kColP = 192, kColDK = 256, kColDV = 384;
  static_assert(kSmemBytes <= 232448, "shared memory budget");
};

struct Bwd128Params {
  const float* lse;    // [B, H, S] natural log
  const float* delta;  // [B, H, S]
  void* dqkv;          // [B*S, lddq] bf16 interleaved [H, 3, dr]
  long long lddq;
  int B, H, S;
  int n_kt;            // 128-key tiles per sequence
  int n_qb;            // 64-query blocks per sequence
  int items;
  int dr;              // real head dim (128 or 80)
  float scale, scale_log2;
  Status* status;
};

__global__ void __launch_bounds__(kBwdThreads, 1)
    bwd128_kernel(const __grid_constant__ CUtensorMap tmKV, const __grid_constant__ CUtensorMap tmQ,
                  const __grid_constant__ CUtensorMap tmDO, const __grid_constant__ CUtensorMap tmDQ,
                  const __grid_constant__ CUtensorMap tmOut, const __grid_constant__ Bwd128Params p) {
  using C = Bwd128Cfg;
  constexpr int D = C::D;
  constexpr int QS = C::kQStages;
  constexpr int BQ = C::kBQ;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  if ((smem_u32(smem_raw) & 1023u) != 0u) {  // uniform across the CTA
    if (threadIdx.x == 0) report(p.status, kBadArgument, 159, smem_u32(smem_raw));
    return;
  }
  uint8_t* sK = smem_raw;
  uint8_t* sV = sK + C::kKTile;
  uint8_t* sQ = sV + C::kKTile;                  // [QS]
  uint8_t* sdO = sQ + QS * C::kQTile;            // [QS]
  uint8_t* sdSt = sdO + QS * C::kQTile;          // dS^T
  uint8_t* sStg = sdSt + C::kPBytes;             // dQ staging (fp32)
  float* sL = reinterpret_cast<float*>(sStg + C::kStgBytes);  // [2][64] lse (log2 units)
  float* sDel = sL + 2 * BQ;                                    // [2][64]
  uint64_t* bars = reinterpret_cast<uint64_t*>(sDel + 2 * BQ);
  static_assert(QS == 3, "barrier slots below are laid out for three Q/dO stages");
  uint64_t* kv_full = bars + 0;
  uint64_t* kv_staged = bars + 1;  // the item's dK / dV are in the K / V buffers
  uint64_t* qd_full = bars + 2;    // [3]
  uint64_t* qd_empty = bars + 5;   // [3]
  uint64_t* sd_full = bars + 8;
  uint64_t* sd_free = bars + 9;
  uint64_t* pds_full = bars + 10;
  uint64_t* p_free = bars + 11;    // [2] dV done reading P^T buffer
  uint64_t* ds_free = bars + 13;   // dK and dQ^T done reading dS^T
  uint64_t* dq_full = bars + 14;
  uint64_t* dq_free = bars + 15;
  uint64_t* dkv_free = bars + 16;
  uint64_t* drain = bars + 17;
  uint64_t* stage_bar = bars + 18;  // [2]
  uint64_t* stg_free = bars + 20;   // staging tile read by the bulk reduce-adds
  uint64_t* dq_staged = bars + 21;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 22);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(bars + 23);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int bhc = p.B * p.H;

  if (threadIdx.x == 0) {
    mbar_init(kv_full, 1);
    mbar_init(kv_staged, kBwdCompute);
    for (int i = 0; i < QS; ++i) {
      mbar_init(&qd_full[i], 1);
      mbar_init(&qd_empty[i], 1);
    }
    mbar_init(sd_full, 1);
    mbar_init(sd_free, kBwdCompute);
    mbar_init(pds_full, kBwdCompute);
    mbar_init(&p_free[0], 1);
    mbar_init(&p_free[1], 1);
    mbar_init(ds_free, 1);
    mbar_init(dq_full, 1);
    mbar_init(dq_free, 4);
    mbar_init(dkv_free, kBwdCompute);
    mbar_init(drain, 1);
    for (int i = 0; i < 2; ++i) mbar_init(&stage_bar[i], kBwdCompute);
    mbar_init(stg_free, 1);
    mbar_init(dq_staged, 4);
    *abort_flag = 0;
    fence_mbar_init();
    tma_prefetch_desc(&tmKV);
    tma_prefetch_desc(&tmQ);
    tma_prefetch_desc(&tmDO);
    tma_prefetch_desc(&tmDQ);
    tma_prefetch_desc(&tmOut);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, C::kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  pdl_trigger();
  pdl_wait();

  if (warp == 0 && lane == 0) {
    // ------------------------------------------------------------ TMA producer
    int kv_armed = -1;
    int q_armed[QS];
    for (int i = 0; i < QS; ++i) q_armed[i] = -1;
    // Store item ti's dK / dV (staged by the compute warps in the K / V buffers).
    auto store_dkv = [&](int ti) -> bool {
      if (!mbar_wait(kv_staged, static_cast<uint32_t>(ti) & 1u, p.status, 164, abort_flag)) return false;
      const int w = blockIdx.x + ti * gridDim.x;
      const int kt = w / bhc, bh = w % bhc, b = bh / p.H, h = bh % p.H;
#pragma unroll
      for (int c = 0; c < 2; ++c) {
        if (c * 64 >= p.dr) break;
        tma_store_4d(&tmOut, sK + c * 16384, c * 64, 3 * h + 1, kt * 128, b);
        tma_store_4d(&tmOut, sV + c * 16384, c * 64, 3 * h + 2, kt * 128, b);
      }
      bulk_commit_group();
      return true;
    };
    int g = 0, t = 0;
    bool ok = true;
    for (int w = blockIdx.x; w < p.items && ok; w += gridDim.x, ++t) {
      const int kt = w / bhc, bh = w % bhc, b = bh / p.H, h = bh % p.H;
      const uint32_t tph = static_cast<uint32_t>(t) & 1u;
      if (t >= 1) {
        // The previous item's dK / dV leave the K / V buffers before they are reloaded.
        if (!store_dkv(t - 1)) break;
        bulk_wait_read_all();
      }
      mbar_arrive_expect_tx(kv_full, 2 * C::kKTile);
      kv_armed = static_cast<int>(tph);
#pragma unroll
      for (int c = 0; c < 2; ++c) {
        tma_load_4d(&tmKV, kv_full, sK + c * 16384, c * 64, 3 * h + 1, kt * 128, b);
        tma_load_4d(&tmKV, kv_full, sV + c * 16384, c * 64, 3 * h + 2, kt * 128, b);
      }
      for (int i = 2 * kt; i < p.n_qb; ++i, ++g) {
        const int st = g % QS;
        const uint32_t ph = static_cast<uint32_t>(g / QS) & 1u;
        if (!mbar_wait(&qd_empty[st], ph ^ 1u, p.status, 161, abort_flag)) {
          ok = false;
          break;
        }
        mbar_arrive_expect_tx(&qd_full[st], 2 * C::kQTile);
        q_armed[st] = static_cast<int>(ph);
#pragma unroll
        for (int c = 0; c < 2; ++c) {
          tma_load_4d(&tmQ, &qd_full[st], sQ + st * C::kQTile + c * C::kQChunk, c * 64, 3 * h, i * BQ, b);
          tma_load_4d(&tmDO, &qd_full[st], sdO + st * C::kQTile + c * C::kQChunk, c * 64, h, i * BQ, b);
        }
      }
    }
    if (ok && t >= 1) store_dkv(t - 1);
    bulk_wait_all();
    if (kv_armed >= 0) mbar_wait(kv_full, static_cast<uint32_t>(kv_armed), p.status, 162, nullptr);
    for (int i = 0; i < QS; ++i)
      if (q_armed[i] >= 0) mbar_wait(&qd_full[i], static_cast<uint32_t>(q_armed[i]), p.status, 163, nullptr);
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer (whole warp, elected lane issues)
    constexpr uint32_t idS = idesc_bf16_f32(128, BQ, false, false);  // S^T, dP^T
    constexpr uint32_t idKV = idesc_bf16_f32(128, D, false, true);   // dK, dV: B (Q, dO) MN-major
    constexpr uint32_t idQT = idesc_bf16_f32(D, BQ, true, true);     // dQ^T: A (K^T), B (dS^T) MN-major
    const uint64_t dK_k = sdesc_sw128(smem_u32(sK), 16, 1024);
    const uint64_t dK_mn = sdesc_sw128(smem_u32(sK), 16384, 1024);
    const uint64_t dV_k = sdesc_sw128(smem_u32(sV), 16, 1024);
    const uint64_t dQ_k = sdesc_sw128(smem_u32(sQ), 16, 1024);
    const uint64_t dQ_mn = sdesc_sw128(smem_u32(sQ), C::kQChunk, 1024);
    const uint64_t ddO_k = sdesc_sw128(smem_u32(sdO), 16, 1024);
    const uint64_t ddO_mn = sdesc_sw128(smem_u32(sdO), C::kQChunk, 1024);
    const uint64_t ddS_k = sdesc_sw128(smem_u32(sdSt), 16, 1024);
    const uint64_t ddS_mn = sdesc_sw128(smem_u32(sdSt), 16384, 1024);
    constexpr uint32_t kQT16 = C::kQTile >> 4;
    int g = 0, t = 0;
    bool ok = true;
    auto issue_scores = [&](int gg) -> bool {
      const int st = gg % QS;
      if (!mbar_wait(&qd_full[st], static_cast<uint32_t>(gg / QS) & 1u, p.status, 170, abort_flag) ||
          !mbar_wait(sd_free, (static_cast<uint32_t>(gg) & 1u) ^ 1u, p.status, 171, abort_flag))
        return false;
      tc_fence_after();
      const uint64_t q0 = dQ_k + st * kQT16, o0 = ddO_k + st * kQT16;
#pragma unroll
      for (int kk = 0; kk < D / 16; ++kk) {
        const uint32_t offk = ((kk >> 2) * 16384 + (kk & 3) * 32) >> 4;
        const uint32_t offq = ((kk >> 2) * C::kQChunk + (kk & 3) * 32) >> 4;
        umma_bf16_ss_elect(tmem + C::kColS, dK_k + offk, q0 + offq, idS, kk > 0 ? 1u : 0u);
        umma_bf16_ss_elect(tmem + C::kColDP, dV_k + offk, o0 + offq, idS, kk > 0 ? 1u : 0u);
      }
      umma_commit_elect(sd_full);
      return true;
    };
    for (int w = blockIdx.x; w < p.items && ok; w += gridDim.x, ++t) {
      const int kt = w / bhc;
      const int n = p.n_qb - 2 * kt;
      if (!mbar_wait(kv_full, static_cast<uint32_t>(t) & 1u, p.status, 172, abort_flag)) break;
      if (!issue_scores(g)) break;
      for (int u = 0; u < n; ++u, ++g) {
        const int st = g % QS;
        const int pb = g & 1;
        // The next block's score products go first once their Q / dO tile has landed;
        // if this block's P / dS arrive before that, this block's products go first.
        bool scores_after = false;
        if (u + 1 < n) {
          const int st1 = (g + 1) % QS;
          const uint64_t t0 = globaltimer_ns();
          for (uint32_t it = 0;; ++it) {
            if (mbar_test_wait(&qd_full[st1], static_cast<uint32_t>((g + 1) / QS) & 1u) &&
                mbar_test_wait(sd_free, (static_cast<uint32_t>(g + 1) & 1u) ^ 1u))
              break;
            if (mbar_test_wait(pds_full, static_cast<uint32_t>(g) & 1u)) {
              scores_after = true;
              break;
            }
            if ((it & 63u) == 63u && (*abort_flag || globaltimer_ns() - t0 > kPipelineTimeoutNs)) {
              if (!*abort_flag) {
                report(p.status, kTimeoutPipeline, 177, 0);
                *abort_flag = 1;
              }
              ok = false;
              break;
            }
          }
          if (!ok) break;
          if (!scores_after && !issue_scores(g + 1)) {
            ok = false;
            break;
          }
        }
        if (!mbar_wait(pds_full, static_cast<uint32_t>(g) & 1u, p.status, 173, abort_flag)) {
          ok = false;
          break;
        }
        if (u == 0 && !mbar_wait(dkv_free, (static_cast<uint32_t>(t) & 1u) ^ 1u, p.status, 174, abort_flag)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint64_t qmn = dQ_mn + st * kQT16, omn = ddO_mn + st * kQT16;
        const uint32_t acc0 = u > 0 ? 1u : 0u;
#pragma unroll
        for (int kk = 0; kk < BQ / 16; ++kk)
          umma_bf16_ss_elect(tmem + C::kColDK, ddS_k + ((kk * 32) >> 4), qmn + kk * 128, idKV, (acc0 | kk) ? 1u : 0u);
        if (!mbar_wait(dq_free, (static_cast<uint32_t>(g) & 1u) ^ 1u, p.status, 175, abort_flag)) {
          ok = false;
          break;
        }
        tc_fence_after();
#pragma unroll
        for (int kk = 0; kk < 128 / 16; ++kk)
          umma_bf16_ss_elect(tmem + C::kColDQ, dK_mn + kk * 128, ddS_mn + kk * 128, idQT, kk > 0 ? 1u : 0u);
        umma_commit_elect(ds_free);
        umma_commit_elect(dq_full);
        // dV += P^T dO with P^T from TMEM buffer pb (8 columns per 16 queries).
#pragma unroll
        for (int kk = 0; kk < BQ / 16; ++kk)
          umma_bf16_ts_elect(tmem + C::kColDV, tmem + C::kColP + static_cast<uint32_t>(pb * 32 + kk * 8), omn + kk * 128,
                             idKV, (acc0 | kk) ? 1u : 0u);
        umma_commit_elect(&qd_empty[st]);
        umma_commit_elect(&p_free[pb]);
        if (scores_after && !issue_scores(g + 1)) {
          ok = false;
          break;
        }
      }
      if (!ok) break;
    }
    umma_commit_elect(drain);
    mbar_wait(drain, 0, p.status, 176, nullptr);
  } else if (warp >= 2 && warp < 2 + kBwdCompute) {
    // ------------------------------------------------------------ compute (thread = key row)
    const int quarter = warp & 3;
    const int half = (warp - 2) >> 2;  // query columns [32*half, 32*half + 32) of the block
    const int krow = quarter * 32 + lane;
    const uint32_t lane_base = static_cast<uint32_t>(quarter * 32) << 16;
    const int ct = threadIdx.x - 64;  // 0..255: 0..63 stage lse, 64..127 delta
    // The prefetch walks this CTA's blocks with a row pointer per item (one integer
    // division per item, none per block); the value is loaded a block before it is staged
    // (threads 128.. load a value they never stage).
    const float* const src = ct < 64 ? p.lse : p.delta;
    auto row_of = [&](int w_) -> const float* { return src + static_cast<long long>(w_ % bhc) * p.S; };
    auto load_raw = [&](const float* row, int i_) -> float { return row[min(i_ * BQ + (ct & 63), p.S - 1)]; };
    auto stage = [&](int gg, int i_, float raw) {
      if (ct < 128) {
        const int q = i_ * BQ + (ct & 63);
        const float v = ct < 64 ? (q < p.S ? raw * 1.4426950408889634f : INFINITY) : (q < p.S ? raw : 0.f);
        (ct < 64 ? sL : sDel)[(gg & 1) * BQ + (ct & 63)] = v;
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&stage_bar[gg & 1]);
    };
    // Advance (w_, i_, row) to the next block of this CTA's work list (w_ = -1 past the end).
    auto next_block = [&](int& w_, int& i_, const float*& row) {
      if (i_ + 1 < p.n_qb) {
        ++i_;
      } else if (w_ + static_cast<int>(gridDim.x) < p.items) {
        w_ += static_cast<int>(gridDim.x);
        i_ = 2 * (w_ / bhc);
        row = row_of(w_);
      } else {
        w_ = -1;
      }
    };
    float pre = 0.f;
    int pre_w = -1, pre_i = 0;
    const float* pre_row = src;
    if (static_cast<int>(blockIdx.x) < p.items) {
      pre_w = blockIdx.x;
      pre_i = 2 * (pre_w / bhc);
      pre_row = row_of(pre_w);
      stage(0, pre_i, load_raw(pre_row, pre_i));
      next_block(pre_w, pre_i, pre_row);
      pre = load_raw(pre_row, pre_i);  // unconditional (a valid row): no select on the loaded value
    }
    int g = 0;
    bool ok = true;
    for (int w = blockIdx.x; w < p.items && ok; w += gridDim.x) {
      const int kt = w / bhc;
      const int n = p.n_qb - 2 * kt;
      for (int u = 0; u < n; ++u, ++g) {
        if (!mbar_wait(&stage_bar[g & 1], static_cast<uint32_t>(g >> 1) & 1u, p.status, 179, abort_flag)) {
          ok = false;
          break;
        }
        const float* L = sL + (g & 1) * BQ + half * 32;
        const float* Dl = sDel + (g & 1) * BQ + half * 32;
        if (!mbar_wait(sd_full, static_cast<uint32_t>(g) & 1u, p.status, 180, abort_flag)) {
          ok = false;
          break;
        }
        tc_fence_after();
        uint32_t sv[32], dv[32];
        tmem_ld_32x32b_x32(tmem + lane_base + C::kColS + static_cast<uint32_t>(half * 32), sv);
        tmem_ld_32x32b_x32(tmem + lane_base + C::kColDP + static_cast<uint32_t>(half * 32), dv);
        tmem_ld_wait();
        // S^T and dP^T in registers: the next block's score products may overwrite them.
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(sd_free);
        // Diagonal: query q_abs < key k_abs is masked; only the first two blocks can hold such pairs.
        const int qoff = (2 * kt + u) * BQ + half * 32 - (kt * 128 + krow);  // q_abs - k_abs at column 0
        uint32_t pp[16], dd[16];
        float4 l4, d4;  // lse / delta of four queries (one 16-byte broadcast load each)
#pragma unroll
        for (int e = 0; e < 32; e += 2) {
          if ((e & 3) == 0) {
            l4 = *reinterpret_cast<const float4*>(L + e);
            d4 = *reinterpret_cast<const float4*>(Dl + e);
          }
          const float la = (e & 3) ? l4.z : l4.x, lb = (e & 3) ? l4.w : l4.y;
          const float da = (e & 3) ? d4.z : d4.x, db = (e & 3) ? d4.w : d4.y;
          float p0 = ex2(fmaf(__uint_as_float(sv[e]), p.scale_log2, -la));
          float p1 = ex2(fmaf(__uint_as_float(sv[e + 1]), p.scale_log2, -lb));
          if (u < 2) {
            if (qoff + e < 0) p0 = 0.f;
            if (qoff + e + 1 < 0) p1 = 0.f;
          }
          const float g0 = p0 * (__uint_as_float(dv[e]) - da);
          const float g1 = p1 * (__uint_as_float(dv[e + 1]) - db);
          pp[e >> 1] = pack_bf16x2(p0, p1);
          dd[e >> 1] = pack_bf16x2(g0, g1);
        }
        // dV of block g-2 is done with this P^T buffer; dK / dQ^T of block g-1 with dS^T.
        if ((g >= 2 && !mbar_wait(&p_free[g & 1], (static_cast<uint32_t>(g >> 1) & 1u) ^ 1u, p.status, 181,
                                  abort_flag)) ||
            (g >= 1 && !mbar_wait(ds_free, static_cast<uint32_t>(g - 1) & 1u, p.status, 182, abort_flag))) {
          ok = false;
          break;
        }
        // P^T to TMEM buffer g & 1 (16 columns = these 32 queries), dS^T to shared memory.
        tc_fence_after();
        tmem_st_32x32b_x16(tmem + lane_base + C::kColP + static_cast<uint32_t>((g & 1) * 32 + half * 16), pp);
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          const uint32_t off = sw128_off(krow, half * 4 + k);
          asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(smem_u32(sdSt + off)), "r"(dd[4 * k]),
                       "r"(dd[4 * k + 1]), "r"(dd[4 * k + 2]), "r"(dd[4 * k + 3])
                       : "memory");
        }
        tmem_st_wait();
        fence_proxy_async_smem();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(pds_full);
        // Stage the next block's lse/delta (its buffer is free: see the waits above), off
        // the path to the P/dS hand-off.
        if (pre_w >= 0) {
          stage(g + 1, pre_i, pre);
          next_block(pre_w, pre_i, pre_row);
          pre = load_raw(pre_row, pre_i);
        }
      }
      if (!ok) break;
      // dV of the last block done: dK and dV of this key tile are final and every product
      // that read K or V has completed.  Stage them (bf16, the 128B-swizzled layout of the
      // K / V tiles: half 0 dK into the K buffer, half 1 dV into the V buffer) for the
      // TMA warp's bulk tensor stores, which clip columns past dr and rows past S.
      if (!mbar_wait(&p_free[(g - 1) & 1], static_cast<uint32_t>((g - 1) >> 1) & 1u, p.status, 183, abort_flag)) break;
      tc_fence_after();
      const float sc = half == 0 ? p.scale : 1.f;
      const uint32_t colx = half == 0 ? C::kColDK : C::kColDV;
      uint8_t* stg = half == 0 ? sK : sV;
#pragma unroll
      for (int c = 0; c < D / 32; ++c) {
        uint32_t o[32];
        tmem_ld_32x32b_x32(tmem + lane_base + colx + c * 32, o);
        tmem_ld_wait();
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          uint8_t* dst = stg + (c >> 1) * 16384 + sw128_off(krow, (c & 1) * 4 + k);
          asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(smem_u32(dst)),
                       "r"(pack_bf16x2(__uint_as_float(o[8 * k + 0]) * sc, __uint_as_float(o[8 * k + 1]) * sc)),
                       "r"(pack_bf16x2(__uint_as_float(o[8 * k + 2]) * sc, __uint_as_float(o[8 * k + 3]) * sc)),
                       "r"(pack_bf16x2(__uint_as_float(o[8 * k + 4]) * sc, __uint_as_float(o[8 * k + 5]) * sc)),
                       "r"(pack_bf16x2(__uint_as_float(o[8 * k + 6]) * sc, __uint_as_float(o[8 * k + 7]) * sc))
                       : "memory");
        }
      }
      fence_proxy_async_smem();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) {
        mbar_arrive(dkv_free);
        mbar_arrive(kv_staged);
      }
    }
  } else if (warp >= 2 + kBwdCompute) {
    // ------------------------------------------------------------ dQ drain (thread = head-dim row)
    const int quarter = warp & 3;  // head-dim rows [32*quarter, +32) = staging box `quarter`
    const uint32_t lane_base = static_cast<uint32_t>(quarter * 32) << 16;
    const bool issuer = warp == 2 + kBwdCompute && lane == 0;
    uint8_t* box = sStg + quarter * (BQ * 128);
    int g = 0;
    bool ok = true;
    for (int w = blockIdx.x; w < p.items && ok; w += gridDim.x) {
      const int kt = w / bhc, bh = w % bhc, b = bh / p.H, h = bh % p.H;
      for (int i = 2 * kt; i < p.n_qb; ++i, ++g) {
        if (!mbar_wait(dq_full, static_cast<uint32_t>(g) & 1u, p.status, 185, abort_flag)) {
          ok = false;
          break;
        }
        tc_fence_after();
        uint32_t o[2][32];
        tmem_ld_32x32b_x32(tmem + lane_base + C::kColDQ, o[0]);
        tmem_ld_32x32b_x32(tmem + lane_base + C::kColDQ + 32, o[1]);
        tmem_ld_wait();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(dq_free);
        // The previous block's reduce-adds have read the staging tile.
        if (g >= 1 && !mbar_wait(stg_free, static_cast<uint32_t>(g - 1) & 1u, p.status, 186, abort_flag)) {
          ok = false;
          break;
        }
        // Element (query q, head-dim row quarter*32 + lane) of box `quarter`: row q, 4-byte word
        // `lane` of the 128-byte row, 16-byte chunk swizzled by q % 8.
#pragma unroll
        for (int c = 0; c < 2; ++c)
#pragma unroll
          for (int e = 0; e < 32; ++e) {
            const int q = c * 32 + e;
            const uint32_t off = static_cast<uint32_t>(q * 128 + ((((lane >> 2) ^ (q & 7))) << 4) + (lane & 3) * 4);
            asm volatile("st.shared.b32 [%0], %1;" ::"r"(smem_u32(box + off)), "r"(o[c][e]) : "memory");
          }
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) mbar_arrive(dq_staged);
        if (issuer) {
          if (!mbar_wait(dq_staged, static_cast<uint32_t>(g) & 1u, p.status, 187, abort_flag)) {
            ok = false;
          } else {
#pragma unroll
            for (int bx = 0; bx < 4; ++bx)
              if (bx * 32 < p.dr) tma_reduce_add_4d(&tmDQ, sStg + bx * (BQ * 128), bx * 32, h, i * BQ, b);
            bulk_commit_group();
            bulk_wait_read_all();
            mbar_arrive(stg_free);
          }
        }
        ok = __shfl_sync(0xFFFFFFFFu, ok ? 1 : 0, 0) != 0;
      }
    }
    if (issuer) bulk_wait_all();
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) tmem_dealloc(tmem, C::kTmemCols);
}

}  // namespace attn_tc
}  // namespace md

// ---------------------------------------------------------------------------
// Host side
// ---------------------------------------------------------------------------
namespace {

PFN_cuTensorMapEncodeTiled_v12000 g_encode_attn = nullptr;

bool get_encoder() {
  if (g_encode_attn != nullptr) return true;
  void* fn = nullptr;
  cudaDriverEntryPointQueryResult q;
  if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q) != cudaSuccess ||
      q != cudaDriverEntryPointSuccess || fn == nullptr)
    return false;
  g_encode_attn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
  return true;
}

// [B, S, cols] view of a [B*S, ld] bf16 matrix; box {64 cols, 128 rows, 1}, 128B swizzle.
bool make_map_bsc(CUtensorMap* map, const void* ptr, int B, int S, long long cols, long long ld) {
  cuuint64_t dims[3] = {static_cast<cuuint64_t>(cols), static_cast<cuuint64_t>(S), static_cast<cuuint64_t>(B)};
  cuuint64_t strides[2] = {static_cast<cuuint64_t>(ld) * 2, static_cast<cuuint64_t>(ld) * 2 * S};
  cuuint32_t box[3] = {64, 128, 1};
  cuuint32_t estr[3] = {1, 1, 1};
  return g_encode_attn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(ptr), dims, strides, box, estr,
                       CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                       CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// [B, S, slots, dr] view of a [B*S, ld] bf16 matrix whose rows hold `slots`
// consecutive dr-wide head vectors; box {64, 1, rows, 1}, 128B swizzle.
// Columns dr..63 of the last box read as zero.
bool make_map_bshd(CUtensorMap* map, const void* ptr, int B, int S, int slots, int dr, long long ld, int rows = 128) {
  cuuint64_t dims[4] = {static_cast<cuuint64_t>(dr), static_cast<cuuint64_t>(slots), static_cast<cuuint64_t>(S),
                        static_cast<cuuint64_t>(B)};
  cuuint64_t strides[3] = {static_cast<cuuint64_t>(dr) * 2, static_cast<cuuint64_t>(ld) * 2,
                           static_cast<cuuint64_t>(ld) * 2 * S};
  cuuint32_t box[4] = {64, 1, static_cast<cuuint32_t>(rows), 1};
  cuuint32_t estr[4] = {1, 1, 1, 1};
  return g_encode_attn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 4, const_cast<void*>(ptr), dims, strides, box, estr,
                       CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                       CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// [B, S, cols] view of a [B*S, ld] fp32 matrix; box {32 cols, 128 rows, 1}, 128B swizzle.
bool make_map_f32_bsc(CUtensorMap* map, const void* ptr, int B, int S, long long cols, long long ld) {
  cuuint64_t dims[3] = {static_cast<cuuint64_t>(cols), static_cast<cuuint64_t>(S), static_cast<cuuint64_t>(B)};
  cuuint64_t strides[2] = {static_cast<cuuint64_t>(ld) * 4, static_cast<cuuint64_t>(ld) * 4 * S};
  cuuint32_t box[3] = {32, 128, 1};
  cuuint32_t estr[3] = {1, 1, 1};
  return g_encode_attn(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 3, const_cast<void*>(ptr), dims, strides, box, estr,
                       CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                       CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// [B, S, H, dr] view of a [B*S, ld] fp32 matrix (head h at columns h*dr); box {32, 1, rows, 1},
// 128B swizzle.  Reduce-adds clip columns past dr and rows past S.
bool make_map_f32_bshd(CUtensorMap* map, const void* ptr, int B, int S, int H, int dr, long long ld, int rows) {
  cuuint64_t dims[4] = {static_cast<cuuint64_t>(dr), static_cast<cuuint64_t>(H), static_cast<cuuint64_t>(S),
                        static_cast<cuuint64_t>(B)};
  cuuint64_t strides[3] = {static_cast<cuuint64_t>(dr) * 4, static_cast<cuuint64_t>(ld) * 4,
                           static_cast<cuuint64_t>(ld) * 4 * S};
  cuuint32_t box[4] = {32, 1, static_cast<cuuint32_t>(rows), 1};
  cuuint32_t estr[4] = {1, 1, 1, 1};
  return g_encode_attn(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, const_cast<void*>(ptr), dims, strides, box, estr,
                       CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                       CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

int g_sms = 0;
long long* g_trace = nullptr;  // device buffer set by md_attn_trace_enable (analysis only)

template <int D>
int fwd_tc_launch(const void* qkv, long long ldq, void* out, long long ldo, float* lse, int B, int H, int S,
                  float scale, void* status, cudaStream_t st, int dr = D) {
  using C = md::attn_tc::FwdCfg<D>;
  if (!get_encoder()) return -3;
  // Loads read Q/K/V in place; the output tiles are stored through a second map
  // (rows past S and, for dr < D, columns past dr are clipped by the store).
  CUtensorMap tm, to;
  if (dr == D) {
    if (!make_map_bsc(&tm, qkv, B, S, 3LL * H * D, ldq) || !make_map_bsc(&to, out, B, S, 1LL * H * D, ldo)) return -4;
  } else {
    if (dr % 8 || dr > D || !make_map_bshd(&tm, qkv, B, S, 3 * H, dr, ldq) ||
        !make_map_bshd(&to, out, B, S, H, dr, ldo))
      return -4;
  }
  if (g_sms == 0) {
    int dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&g_sms, cudaDevAttrMultiProcessorCount, dev);
  }
  md::attn_tc::FwdParams p;
  p.lse = lse;
  p.B = B;
  p.H = H;
  p.S = S;
  p.n_qt = (S + md::attn_tc::kBM - 1) / md::attn_tc::kBM;
  p.items = p.n_qt * B * H;
  p.scale_log2 = scale * 1.4426950408889634f;
  p.status = reinterpret_cast<md::Status*>(status);
  p.dr = dr;
  p.trace = g_trace;
  auto k = g_trace != nullptr ? md::attn_tc::fwd_kernel<D, true> : md::attn_tc::fwd_kernel<D, false>;
  cudaError_t e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, C::kSmemBytes);
  if (e != cudaSuccess) return static_cast<int>(e);
  const int slots = g_sms * C::kCtasPerSm;
  const int grid = p.items < slots ? p.items : slots;
  md::launch_pdl(k, grid, dim3(C::kThreads), C::kSmemBytes, st, tm, to, p);
  return static_cast<int>(cudaGetLastError());
}


template <int D>
int bwd_tc_launch(const void* qkv, long long ldq, const void* dout, long long lddo, const float* lse,
                  const float* delta, float* dqacc, long long ldacc, void* dqkv, long long lddq, int B, int H, int S,
                  float scale, void* status, cudaStream_t st) {
  using C = md::attn_tc::BwdCfg<D>;
  if (!get_encoder()) return -3;
  CUtensorMap tq, tdo, tdq, tout;
  if (!make_map_bsc(&tq, qkv, B, S, 3LL * H * D, ldq) || !make_map_bsc(&tdo, dout, B, S, 1LL * H * D, lddo) ||
      !make_map_f32_bsc(&tdq, dqacc, B, S, 1LL * H * D, ldacc) || !make_map_bsc(&tout, dqkv, B, S, 3LL * H * D, lddq))
    return -4;
  if (g_sms == 0) {
    int dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&g_sms, cudaDevAttrMultiProcessorCount, dev);
  }
  md::attn_tc::BwdParams p;
  p.lse = lse;
  p.delta = delta;
  p.dqacc = dqacc;
  p.ldacc = ldacc;
  p.dqkv = dqkv;
  p.lddq = lddq;
  p.B = B;
  p.H = H;
  p.S = S;
  p.n_t = (S + 127) / 128;
  p.items = p.n_t * B * H;
  p.scale = scale;
  p.scale_log2 = scale * 1.4426950408889634f;
  static const int flags = [] {
    const char* v = getenv("MINIDIST_ATTN_BWD_FLAGS");
    return v ? atoi(v) : 0;
  }();
  p.flags = flags;
  p.status = reinterpret_cast<md::Status*>(status);
  p.trace = g_trace;
  auto k = g_trace != nullptr ? md::attn_tc::bwd_kernel<D, true> : md::attn_tc::bwd_kernel<D, false>;
  cudaError_t e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, C::kSmemBytes);
  if (e != cudaSuccess) return static_cast<int>(e);
  const int grid = p.items < g_sms ? p.items : g_sms;
  md::launch_pdl(k, grid, dim3(md::attn_tc::kBwdThreads), C::kSmemBytes, st, tq, tdo, tdq, tout, p);
  return static_cast<int>(cudaGetLastError());
}

// head_dim 128 (dr = 128) or 80 (dr = 80, zero-padded boxes): bwd128_kernel.
int bwd128_tc_launch(const void* qkv, long long ldq, const void* dout, long long lddo, const float* lse,
                     const float* delta, float* dqacc, long long ldacc, void* dqkv, long long lddq, int B, int H,
                     int S, int dr, float scale, void* status, cudaStream_t st) {
  using C = md::attn_tc::Bwd128Cfg;
  if (!get_encoder()) return -3;
  if (dr % 8 || dr > 128 || dr < 72 || ldacc != static_cast<long long>(H) * dr) return -2;
  CUtensorMap tkv, tq, tdo, tdq, tout;
  if (!make_map_bshd(&tkv, qkv, B, S, 3 * H, dr, ldq, 128) || !make_map_bshd(&tq, qkv, B, S, 3 * H, dr, ldq, 64) ||
      !make_map_bshd(&tdo, dout, B, S, H, dr, lddo, 64) || !make_map_f32_bshd(&tdq, dqacc, B, S, H, dr, ldacc, 64) ||
      !make_map_bshd(&tout, dqkv, B, S, 3 * H, dr, lddq, 128))
    return -4;
  if (g_sms == 0) {
    int dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&g_sms, cudaDevAttrMultiProcessorCount, dev);
  }
  md::attn_tc::Bwd128Params p;
  p.lse = lse;
  p.delta = delta;
  p.dqkv = dqkv;
  p.lddq = lddq;
  p.B = B;
  p.H = H;
  p.S = S;
  p.n_kt = (S + 127) / 128;
  p.n_qb = (S + 63) / 64;
  p.items = p.n_kt * B * H;
  p.dr = dr;
  p.scale = scale;
  p.scale_log2 = scale * 1.4426950408889634f;
  p.status = reinterpret_cast<md::Status*>(status);
  auto k = md::attn_tc::bwd128_kernel;
  cudaError_t e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, C::kSmemBytes);
  if (e != cudaSuccess) return static_cast<int>(e);
  const int grid = p.items < g_sms ? p.items : g_sms;
  md::launch_pdl(k, grid, dim3(md::attn_tc::kBwdThreads), C::kSmemBytes, st, tkv, tq, tdo, tdq, tout, p);
  return static_cast<int>(cudaGetLastError());
}

}  // namespace

extern "C" {

// Main pass of the tcgen05 attention backward (head_dim 64, 80 or 128): dK, dV into dqkv
// and dQ (unscaled) added into the zeroed fp32 accumulator dqacc [B*S, ldacc].
// delta [B, H, S] = rowsum(dO * O) must be ready.  attention.cu's
// md_attn_bwd_tc wraps this with the delta and dQ conversion steps.
int md_attn_bwd_tc_main(const void* qkv, long long ldq, const void* dout, long long lddo, const float* lse,
                        const float* delta, float* dqacc, long long ldacc, void* dqkv, long long lddq, int B, int H,
                        int S, int D, float scale, void* status, cudaStream_t st) {
  if (D == 64)
    return bwd_tc_launch<64>(qkv, ldq, dout, lddo, lse, delta, dqacc, ldacc, dqkv, lddq, B, H, S, scale, status, st);
  if (D == 80 || D == 128)
    return bwd128_tc_launch(qkv, ldq, dout, lddo, lse, delta, dqacc, ldacc, dqkv, lddq, B, H, S, D, scale, status, st);
  return -2;
}

// Performance analysis: record clock64() hand-off timestamps of CTA 0 of the
// backward kernel into a [64][32] device buffer (enable=1), read them back
// into host memory (md_attn_trace_read), or switch recording off (enable=0).
int md_attn_trace_enable(int enable) {
  if (enable && g_trace == nullptr) {
    if (cudaMalloc(&g_trace, 64 * 32 * sizeof(long long)) != cudaSuccess) return -1;
    cudaMemset(g_trace, 0, 64 * 32 * sizeof(long long));
  }
  if (!enable && g_trace != nullptr) {
    cudaFree(g_trace);
    g_trace = nullptr;
  }
  return 0;
}
int md_attn_trace_read(long long* host) {
  if (g_trace == nullptr) return -1;
  return static_cast<int>(cudaMemcpy(host, g_trace, 64 * 32 * sizeof(long long), cudaMemcpyDeviceToHost));
}

// tcgen05 causal attention forward; same layouts as md_attn_fwd (attention.cu).
// head_dim 64 or 128; status: md::Status word the kernel reports a timed-out
// wait into (may be null).
int md_attn_fwd_tc(const void* qkv, long long ldq, void* out, long long ldo, float* lse, int B, int H, int S, int D,
                   float scale, void* status, cudaStream_t st) {
  if (B <= 0 || H <= 0 || S <= 0 || (reinterpret_cast<uintptr_t>(qkv) & 15) || (reinterpret_cast<uintptr_t>(out) & 15) ||
      (ldq % 8) || (ldo % 8))
    return -1;
  switch (D) {
    case 64: return fwd_tc_launch<64>(qkv, ldq, out, ldo, lse, B, H, S, scale, status, st);
    case 128: return fwd_tc_launch<128>(qkv, ldq, out, ldo, lse, B, H, S, scale, status, st);
    // d = 80 (the 2.7B model): the D = 128 kernel on zero-padded boxes.
    case 80: return fwd_tc_launch<128>(qkv, ldq, out, ldo, lse, B, H, S, scale, status, st, 80);
    default: return -2;
  }
}

}  // extern "C"
