"""Collectives of the fused B200 path.

* :class:`FusedBucketReducer` — DDP's bucket reducer on peer memory: the
  gradient buckets live in a :class:`~minidist.parallel.symm.SymmBuffer`
  (every parameter's ``.grad`` is a view into it), and each bucket is averaged
  by one ``md_ar_bucket_kernel`` launch (1/W scale + reduce-scatter +
  all-gather over NVLink, csrc/symm.cu) on a side stream, ordered after the
  compute stream with CUDA events.  Launch order is bucket 0, 1, 2, ... on
  every rank, as with NCCL.
* :func:`gemm_all_reduce` — the row-parallel linear with its all-reduce fused
  into the GEMM kernel (``md_gemm_ar``, peer memory); :func:`all_reduce_` —
  NCCL all-reduce of a bf16 activation (gradient) for the other TP sites.

Byte accounting goes to :data:`minidist.comm.comm_stats` with the same
formulas as the NCCL path.
"""

from __future__ import annotations

import ctypes
import os

import torch

from .. import comm
from ..ops import _native as nat
from ..ops import gemm as G
from . import symm

_MAXW = 8
_DDP_CHANNEL = 0


class ArParams(ctypes.Structure):
    """Mirror of ``struct MdArParams`` (csrc/symm.cu)."""

    _fields_ = [
        ("bufs", ctypes.c_void_p * _MAXW),
        ("flags", ctypes.c_void_p * _MAXW),
        ("offset", ctypes.c_longlong),
        ("n", ctypes.c_longlong),
        ("world", ctypes.c_int),
        ("rank", ctypes.c_int),
        ("scale", ctypes.c_float),
        ("channel", ctypes.c_int),
        ("timeout_ns", ctypes.c_ulonglong),
        ("status", ctypes.c_void_p),
    ]


nat.declare("md_allreduce", "i:pip")


_NVTX = os.environ.get("MINIDIST_NVTX", "0") not in ("0", "", "false", "no")


class _Range:
    """NVTX range named like the fused kernel it brackets (``MINIDIST_NVTX=1``; free otherwise), so
    timelines attribute peer-memory collectives even where kernel names are not shown."""

    __slots__ = ("name",)

    def __init__(self, name: str):
        self.name = name

    def __enter__(self):
        if _NVTX:
            torch.cuda.nvtx.range_push(self.name)

    def __exit__(self, *exc):
        if _NVTX:
            torch.cuda.nvtx.range_pop()


_AR_CTA_CAP = int(os.environ.get("MINIDIST_AR_CTAS", "0"))


def _timeout_ns() -> int:
    return int(float(os.environ.get("MINIDIST_PEER_TIMEOUT_S", "60")) * 1e9)


def allreduce_fp32_(buf: symm.SymmBuffer, comm_: symm.Communicator, elem_offset: int, n: int, scale: float,
                    channel: int, stream: torch.cuda.Stream | None = None) -> None:
    """In-place ``scale * sum over ranks`` of ``n`` fp32 elements at ``elem_offset`` of ``buf`` on every rank."""
    lib = nat.lib()
    p = ArParams()
    for r in range(buf.world):
        p.bufs[r] = buf.ptrs[r]
        p.flags[r] = buf.flag_ptrs[r]
    p.offset, p.n = elem_offset, n
    p.world, p.rank = buf.world, buf.rank
    p.scale = scale
    p.channel = channel
    p.timeout_ns = _timeout_ns()
    p.status = nat.status_ptr()
    ctas = lib.md_allreduce_ctas(n, buf.world)
    if _AR_CTA_CAP > 0:  # MINIDIST_AR_CTAS: fewer CTAs leave more SMs to the backward it overlaps
        ctas = max(1, min(ctas, _AR_CTA_CAP))
    with _Range("md_ar_bucket"):
        nat.check(lib.md_allreduce(ctypes.byref(p), ctas, ctypes.c_void_p(nat.stream_ptr(stream))), "md_allreduce")


class FusedBucketReducer:
    """DDP reducer whose buckets are reduced by the peer-memory kernel."""

    name = "fused-nvlink"

    def __init__(self, ddp, comm_: symm.Communicator):
        self.comm = comm_
        self.world = ddp.world_size
        self.stream = torch.cuda.Stream()
        self.buf: symm.SymmBuffer | None = None
        self.base = 0

    def allocate(self, numel: int, dtype, device) -> torch.Tensor:
        if dtype != torch.float32:
            raise TypeError("fused bucket reduction expects fp32 gradients")
        self.buf = symm.SymmBuffer(self.comm.group, numel * 4)
        t = self.buf.view(torch.float32, 0, numel)
        self.base = t.data_ptr()
        return t

    def launch(self, b) -> None:
        cur = torch.cuda.current_stream()
        if os.environ.get("MINIDIST_DEBUG_SYNC") == "1":
            torch.cuda.synchronize()
        self.stream.wait_stream(cur)
        off = (b.buffer.data_ptr() - self.base) // 4
        allreduce_fp32_(self.buf, self.comm, off, b.numel, 1.0 / self.world, _DDP_CHANNEL, self.stream)
        ev = torch.cuda.Event()
        ev.record(self.stream)
        b.work = ev
        nbytes = b.payload_numel * 4
        comm.comm_stats.add("all_reduce", nbytes, comm.bus_bytes("all_reduce", nbytes, self.world))

    def wait(self, b) -> None:
        if b.work is not None:
            torch.cuda.current_stream().wait_event(b.work)


def make_bucket_reducer(ddp, required: bool = False):
    """A :class:`FusedBucketReducer` when peer memory works for the DDP group, else ``None``."""
    group = ddp.process_group
    ranks = list(range(comm.get_world_size())) if group is None else torch.distributed.get_process_group_ranks(group)
    c = symm.communicator(group, ranks)
    if c is None:
        if required:
            raise RuntimeError("MINIDIST_DDP_REDUCER=fused but peer memory is unavailable for this group")
        return None
    return FusedBucketReducer(ddp, c)


# ---------------------------------------------------------------------------
# Tensor parallel
# ---------------------------------------------------------------------------


def all_reduce_(t: torch.Tensor, group) -> torch.Tensor:
    """NCCL all-reduce (sum) of ``t`` in place: the fallback for the tensor-parallel sites whose
    peer-memory kernel is unavailable (no shared node, ``MINIDIST_TP_FUSED=0``, unsupported shape)."""
    comm.all_reduce(t, group=group)
    return t


_EMB_CHANNEL = 7


class EmbTpParams(ctypes.Structure):
    """Mirror of ``struct MdEmbTpParams`` (csrc/symm.cu)."""

    _fields_ = [
        ("wte", ctypes.c_void_p * _MAXW),
        ("flags", ctypes.c_void_p * _MAXW),
        ("world", ctypes.c_int),
        ("rank", ctypes.c_int),
        ("channel", ctypes.c_int),
        ("timeout_ns", ctypes.c_ulonglong),
        ("status", ctypes.c_void_p),
        ("ids", ctypes.c_void_p),
        ("wpe", ctypes.c_void_p),
        ("ldp", ctypes.c_longlong),
        ("out", ctypes.c_void_p),
        ("ldo", ctypes.c_longlong),
        ("ldw", ctypes.c_longlong),
        ("vocab_rows", ctypes.c_longlong),
        ("M", ctypes.c_int),
        ("S", ctypes.c_int),
        ("C", ctypes.c_int),
    ]


nat.declare("md_embed_tp", "i:pip")


def symmetric_bf16_shadow(c: symm.Communicator, p: torch.Tensor):
    """Give fp32 parameter ``p`` a bf16 shadow that lives in symmetric memory (peers can read
    it); returns ``(shadow, buffer)``.  The shadow is refreshed like any other (a cast when
    ``p`` changed, or in place by :class:`~minidist.optim.FusedAdamW`).  The first call is
    collective over ``c``'s group: every rank registers its tables in the same order."""
    from ..models import fused_gpt as F

    buf = getattr(p, "_md_symm_shadow_buf", None)
    if buf is None:
        tables = c.__dict__.setdefault("_shadow_tables", [])
        buf = c.buffer(f"tp_table_{len(tables)}", p.numel() * 2)
        tables.append(buf)
        setattr(p, F._SHADOW, buf.view(torch.bfloat16, 0, p.numel()).view(p.shape))
        setattr(p, F._SHADOW_VER, None)  # force the first refresh
        p._md_symm_shadow_buf = buf
    return F.bf16_weight(p), buf


def embedding_tp(ids: torch.Tensor, wte: torch.Tensor, wpe_bf16: torch.Tensor, group) -> torch.Tensor | None:
    """Vocab-parallel embedding forward ``wte[ids] + wpe[s]`` (bf16 ``[B*S, C]``) read straight from
    the owning rank's table shard over NVLink (``md_embed_tp``); ``None`` when peer memory is
    unavailable for ``group`` (the caller does the masked lookup + NCCL all-reduce)."""
    if not _tp_fused_enabled() or wte.dtype != torch.float32:
        return None
    c = _group_comm(group)
    if c is None or wte.shape[1] % 8:
        return None
    shadow, buf = symmetric_bf16_shadow(c, wte)
    B, S = ids.shape
    M, C = B * S, shadow.shape[1]
    ids_c = ids.reshape(-1)
    if ids_c.dtype != torch.int64 or not ids_c.is_contiguous():
        ids_c = ids_c.to(torch.int64).contiguous()
    out = torch.empty(M, C, dtype=torch.bfloat16, device=ids.device)
    prm = EmbTpParams()
    for r in range(c.world):
        prm.wte[r], prm.flags[r] = buf.ptrs[r], buf.flag_ptrs[r]
    prm.world, prm.rank, prm.channel = c.world, c.rank, _EMB_CHANNEL
    prm.timeout_ns, prm.status = _timeout_ns(), nat.status_ptr(ids.device)
    prm.ids, prm.wpe, prm.ldp = ids_c.data_ptr(), wpe_bf16.data_ptr(), wpe_bf16.stride(0)
    prm.out, prm.ldo = out.data_ptr(), out.stride(0)
    prm.ldw, prm.vocab_rows = shadow.stride(0), shadow.shape[0]
    prm.M, prm.S, prm.C = M, S, C
    ctas = min(148, max(1, -(-M // 32)))
    with _Range("md_embed_tp"):
        rc = nat.lib().md_embed_tp(ctypes.byref(prm), ctas, ctypes.c_void_p(nat.stream_ptr(None)))
    nat.check(rc, "md_embed_tp")
    # Bytes as the all-reduce it replaces would count them (so CommStats stays comparable).
    n = M * C * 2
    comm.comm_stats.add("all_reduce", n, comm.bus_bytes("all_reduce", n, c.world))
    return out




class TpArParams(ctypes.Structure):
    """Mirror of ``struct MdTpArParams`` (csrc/gemm_sm100.cu)."""

    _fields_ = [
        ("partial", ctypes.c_void_p * _MAXW),
        ("fin", ctypes.c_void_p * _MAXW),
        ("flags", ctypes.c_void_p * _MAXW),
        ("ldp", ctypes.c_longlong),
        ("out", ctypes.c_void_p),
        ("ldo", ctypes.c_longlong),
        ("bias", ctypes.c_void_p),
        ("resid", ctypes.c_void_p),
        ("ldr", ctypes.c_longlong),
        ("world", ctypes.c_int),
        ("rank", ctypes.c_int),
        ("epoch", ctypes.c_uint32),
        ("max_chunks", ctypes.c_int),
        ("timeout_ns", ctypes.c_ulonglong),
        ("trace", ctypes.c_void_p),
        ("claim", ctypes.c_void_p),
    ]


nat.declare("md_gemm_ar", "i:ppp")
_AR_CACHE: dict[int, tuple] = {}


class _LazyFn:
    def __init__(self, name):
        self.name, self.fn = name, None

    def __call__(self, *a):
        if self.fn is None:
            self.fn = getattr(nat.lib(), self.name)
        return self.fn(*a)


_LIB_GEMM_AR = _LazyFn("md_gemm_ar")


def _group_comm(group) -> symm.Communicator | None:
    if not (torch.cuda.is_available() and comm.is_distributed()):
        return None
    ranks = list(range(comm.get_world_size())) if group is None else torch.distributed.get_process_group_ranks(group)
    return symm.communicator(group, ranks)


def _tp_fused_enabled() -> bool:
    return os.environ.get("MINIDIST_TP_FUSED", "1") not in ("0", "false", "no")


def dgrad_all_reduce(dy_local: torch.Tensor, w_local: torch.Tensor, group) -> torch.Tensor:
    """``all_reduce(dy_local @ w_local)`` (bf16): the tensor-parallel ``f`` backward of a
    column-parallel layer (tensor_parallel.py:148-152) fused with its data-gradient GEMM."""
    return gemm_all_reduce(dy_local, w_local, None, None, group, b_mn=True)


def gemm_all_reduce(x_local, w_local, bias, resid, group, b_mn: bool = False):
    """``resid + bias + all_reduce(x_local @ w_local^T)`` (bf16) over the tensor-parallel group.

    On the fused path this is one ``md_gemm_ar`` launch: the GEMM epilogue
    publishes bf16 partial tiles into a symmetric buffer, and comm warps of the
    same persistent kernel reduce the tiles this rank owns over NVLink (bias and
    residual added once, as the reference adds the bias after the reduce,
    tensor_parallel.py:354-368) and copy every other tile from its owner.
    Otherwise: GEMM, NCCL all-reduce, then bias/residual.
    """
    M, K = x_local.shape
    N = w_local.shape[1] if b_mn else w_local.shape[0]
    c = _group_comm(group) if _tp_fused_enabled() else None
    if c is None or c.world not in (2, 4, 8) or N % 8 or x_local.stride(1) != 1 or w_local.stride(1) != 1:
        out = G.linear_dgrad(x_local, w_local) if b_mn else G.linear_fwd(x_local, w_local)
        comm.all_reduce(out, group=group)
        acc = out.float()
        if bias is not None:
            acc += bias
        if resid is not None:
            acc += resid.float()
        res = G.empty_padded(out.shape[0], out.shape[1], device=out.device)
        res.copy_(acc)
        return res
    ldp = N
    chunks = (M + 31) // 32 * ((N + 255) // 256)
    part = c.buffer("tp_partial", M * ldp * 2)
    fin = c.buffer("tp_final", M * ldp * 2)
    flags = c.zeroed_buffer("tp_flags", 2 * chunks * 4)
    out = G.empty_padded(M, N, device=x_local.device)
    # The parameter structs are built once per (buffers, shape) and patched per call.
    key = (id(part), id(fin), id(flags), M, N, K, b_mn)
    st = _AR_CACHE.get(id(c))
    if st is None or st[0] != key:
        ar = TpArParams()
        for r in range(c.world):
            ar.partial[r] = part.ptrs[r]
            ar.fin[r] = fin.ptrs[r]
            ar.flags[r] = flags.ptrs[r]
        ar.ldp = ldp
        ar.world, ar.rank = c.world, c.rank
        ar.max_chunks = flags.nbytes // 8
        ar.timeout_ns = _timeout_ns()
        # {claimed, finished, launches} counters of this rank: one set per communicator for
        # its whole life, since the launch count is the flags' epoch.
        claim = getattr(c, "tp_claim", None)
        if claim is None:
            claim = c.tp_claim = torch.zeros(3, dtype=torch.int32, device=x_local.device)
        ar.claim = claim.data_ptr()
        gp = nat.GemmParams()
        gp.M, gp.N, gp.K = M, N, K
        gp.epi = G.EPI_BF16
        gp.alpha = 1.0
        gp.b_mn_major = int(b_mn)
        gp.status = nat.status_ptr(x_local.device)
        st = (key, ar, gp, ctypes.byref(gp), ctypes.byref(ar), claim)
        _AR_CACHE[id(c)] = st
    _, ar, gp, gp_ref, ar_ref, _ = st
    ar.out, ar.ldo = out.data_ptr(), out.stride(0)
    ar.bias = None if bias is None else bias.data_ptr()
    if resid is not None:
        ar.resid, ar.ldr = resid.data_ptr(), resid.stride(0)
    else:
        ar.resid = None
    gp.A, gp.B = x_local.data_ptr(), w_local.data_ptr()
    gp.lda, gp.ldb = x_local.stride(0), w_local.stride(0)
    with _Range("md_gemm_ar"):
        rc = _LIB_GEMM_AR(gp_ref, ar_ref, ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    if rc != 0:
        nat.check(rc, f"md_gemm_ar(M={M},N={N},K={K})")
    comm.comm_stats.add("all_reduce", M * N * 2, int(2 * (c.world - 1) / c.world * M * N * 2))
    return out


# ---------------------------------------------------------------------------
# FSDP: reduce-scatter (+ AdamW) over peer memory
# ---------------------------------------------------------------------------
_FSDP_CHANNEL = 4


class RsParams(ctypes.Structure):
    """Mirror of ``struct MdRsParams`` (csrc/symm.cu)."""

    _fields_ = [
        ("bufs", ctypes.c_void_p * _MAXW),
        ("flags", ctypes.c_void_p * _MAXW),
        ("offset", ctypes.c_longlong),
        ("shard", ctypes.c_longlong),
        ("world", ctypes.c_int),
        ("rank", ctypes.c_int),
        ("scale", ctypes.c_float),
        ("channel", ctypes.c_int),
        ("timeout_ns", ctypes.c_ulonglong),
        ("status", ctypes.c_void_p),
        ("grad_out", ctypes.c_void_p),
        ("accumulate", ctypes.c_int),
        ("p", ctypes.c_void_p),
        ("m", ctypes.c_void_p),
        ("v", ctypes.c_void_p),
        ("lr", ctypes.c_float),
        ("b1", ctypes.c_float),
        ("b2", ctypes.c_float),
        ("eps", ctypes.c_float),
        ("wd", ctypes.c_float),
        ("bc1", ctypes.c_float),
        ("bc2_sqrt", ctypes.c_float),
        ("p_bf16", ctypes.c_void_p),
    ]


nat.declare("md_rs_shard", "i:pip")


def fsdp_communicator(group) -> symm.Communicator | None:
    """Peer-memory communicator for FSDP's gradient reduce-scatter (``None`` -> NCCL)."""
    if os.environ.get("MINIDIST_FSDP_FUSED", "1") in ("0", "false", "no"):
        return None
    return _group_comm(group)


def fsdp_gather_enabled() -> bool:
    """Peer-memory parameter all-gather for FSDP (env ``MINIDIST_FSDP_GATHER=0`` -> NCCL)."""
    return os.environ.get("MINIDIST_FSDP_GATHER", "1") not in ("0", "false", "no")


def reduce_scatter_shard(buf: symm.SymmBuffer, comm_: symm.Communicator, elem_offset: int, shard: int,
                         grad_out: torch.Tensor | None, accumulate: bool, scale: float,
                         adam: tuple | None = None, p_bf16: torch.Tensor | None = None) -> None:
    """Rank r's slice ``[elem_offset + r*shard, +shard)`` of ``buf`` summed over ranks, times ``scale``,
    into ``grad_out`` (or, with ``adam = (p, m, v, lr, b1, b2, eps, wd, step)``, an AdamW update of ``p``)."""
    prm = RsParams()
    for r in range(comm_.world):
        prm.bufs[r] = buf.ptrs[r]
        prm.flags[r] = buf.flag_ptrs[r]
    prm.offset, prm.shard = elem_offset, shard
    prm.world, prm.rank = comm_.world, comm_.rank
    prm.scale = scale
    prm.channel = _FSDP_CHANNEL
    prm.timeout_ns = _timeout_ns()
    prm.status = nat.status_ptr(buf.device)
    if adam is not None:
        p, m, v, lr, b1, b2, eps, wd, step = adam
        prm.p, prm.m, prm.v = p.data_ptr(), m.data_ptr(), v.data_ptr()
        prm.lr, prm.b1, prm.b2, prm.eps, prm.wd = lr, b1, b2, eps, wd
        prm.bc1 = 1.0 - b1 ** step
        prm.bc2_sqrt = (1.0 - b2 ** step) ** 0.5
        prm.p_bf16 = None if p_bf16 is None else p_bf16.data_ptr()
    else:
        prm.grad_out = grad_out.data_ptr()
        prm.accumulate = int(accumulate)
    # At most 64 CTAs: the reduce-scatter runs beside the backward on the communication stream,
    # and 64 x 512 threads with 2 x W vectors in flight each already saturate NVLink.
    ctas = min(64, max(1, shard // (4 * 512 * 8)))
    with _Range("md_rs_shard"):
        rc = nat.lib().md_rs_shard(ctypes.byref(prm), ctas, ctypes.c_void_p(nat.stream_ptr(None)))
    nat.check(rc, "md_rs_shard")
    n = shard * comm_.world * 4
    comm.comm_stats.add("reduce_scatter", n, int((comm_.world - 1) / comm_.world * n))


# ---------------------------------------------------------------------------
# FSDP: parameter all-gather over peer memory
# ---------------------------------------------------------------------------
_FSDP_AG_CHANNEL = 5


class AgParams(ctypes.Structure):
    """Mirror of ``struct MdAgParams`` (csrc/symm.cu)."""

    _fields_ = [
        ("bufs", ctypes.c_void_p * _MAXW),
        ("flags", ctypes.c_void_p * _MAXW),
        ("offset", ctypes.c_longlong),
        ("shard", ctypes.c_longlong),
        ("world", ctypes.c_int),
        ("rank", ctypes.c_int),
        ("channel", ctypes.c_int),
        ("timeout_ns", ctypes.c_ulonglong),
        ("status", ctypes.c_void_p),
        ("out", ctypes.c_void_p),
        ("out_bf16", ctypes.c_int),
        ("in_bf16", ctypes.c_int),
    ]


nat.declare("md_ag_shards", "i:pip")


def all_gather_shards(buf: symm.SymmBuffer, comm_: symm.Communicator, elem_offset: int, shard: int,
                      out: torch.Tensor, src_bf16: bool = False) -> None:
    """Every rank's shard ``buf[elem_offset : elem_offset + shard]`` into ``out`` (rank r's at
    ``out[r*shard]``), on the current stream: fp32 shards cast to ``out.dtype`` (fp32 or bf16)
    on the way, or with ``src_bf16`` bf16 shards copied into a bf16 ``out``."""
    if out.dtype not in (torch.float32, torch.bfloat16) or out.numel() < shard * comm_.world:
        raise ValueError("all_gather_shards: out must be fp32 / bf16 with world * shard elements")
    if src_bf16 and (out.dtype != torch.bfloat16 or shard % 8 or elem_offset % 8):
        raise ValueError("all_gather_shards: bf16 shards need a bf16 out and 8-element alignment")
    prm = AgParams()
    for r in range(comm_.world):
        prm.bufs[r] = buf.ptrs[r]
        prm.flags[r] = buf.flag_ptrs[r]
    prm.offset, prm.shard = elem_offset, shard
    prm.world, prm.rank = comm_.world, comm_.rank
    prm.channel = _FSDP_AG_CHANNEL
    prm.timeout_ns = _timeout_ns()
    prm.status = nat.status_ptr(buf.device)
    prm.out = out.data_ptr()
    prm.out_bf16 = int(out.dtype == torch.bfloat16)
    prm.in_bf16 = int(src_bf16)
    # One CTA per 64 K output elements, at most 64: the gather overlaps the compute stream.
    ctas = min(64, max(1, shard * comm_.world // 65536))
    with _Range("md_ag_shards"):
        rc = nat.lib().md_ag_shards(ctypes.byref(prm), ctas, ctypes.c_void_p(nat.stream_ptr(None)))
    nat.check(rc, "md_ag_shards")
    n = shard * comm_.world * out.element_size()
    comm.comm_stats.add("all_gather", n, int((comm_.world - 1) / comm_.world * n))
    # (bf16 sources move half the bytes of fp32 ones; the count above is the gathered payload,
    # the reference's accounting for a gather in param_dtype.)


# ---------------------------------------------------------------------------
# Vocab-parallel cross-entropy statistics over peer memory
# ---------------------------------------------------------------------------
_CE_CHANNEL = 6


class CeTpParams(ctypes.Structure):
    """Mirror of ``struct MdCeTpParams`` (csrc/symm.cu)."""

    _fields_ = [
        ("bufs", ctypes.c_void_p * _MAXW),
        ("flags", ctypes.c_void_p * _MAXW),
        ("world", ctypes.c_int),
        ("rank", ctypes.c_int),
        ("channel", ctypes.c_int),
        ("timeout_ns", ctypes.c_ulonglong),
        ("status", ctypes.c_void_p),
        ("tmax", ctypes.c_void_p),
        ("tsum", ctypes.c_void_p),
        ("tiles", ctypes.c_int),
        ("ttgt", ctypes.c_void_p),
        ("M", ctypes.c_int),
        ("lse", ctypes.c_void_p),
        ("loss", ctypes.c_void_p),
    ]


nat.declare("md_ce_tp", "i:pip")


def ce_tp_stats(tmax: torch.Tensor, tsum: torch.Tensor, ttgt: torch.Tensor, group):
    """``(lse, loss_rows)`` of a vocab-parallel cross-entropy from this rank's per-slab statistics
    (``tmax``/``tsum`` ``[tiles, M]``, target logit ``ttgt`` ``[M]``) in one peer-memory kernel,
    or ``None`` when peer memory is unavailable for ``group`` (the caller uses NCCL)."""
    if not _tp_fused_enabled():
        return None
    c = _group_comm(group)
    if c is None:
        return None
    tiles, M = tmax.shape
    buf = c.buffer("tp_ce", 3 * M * 4)
    lse = torch.empty(M, dtype=torch.float32, device=tmax.device)
    loss = torch.empty_like(lse)
    prm = CeTpParams()
    for r in range(c.world):
        prm.bufs[r], prm.flags[r] = buf.ptrs[r], buf.flag_ptrs[r]
    prm.world, prm.rank, prm.channel = c.world, c.rank, _CE_CHANNEL
    prm.timeout_ns, prm.status = _timeout_ns(), nat.status_ptr(tmax.device)
    prm.tmax, prm.tsum, prm.tiles = tmax.data_ptr(), tsum.data_ptr(), tiles
    prm.ttgt, prm.M = ttgt.data_ptr(), M
    prm.lse, prm.loss = lse.data_ptr(), loss.data_ptr()
    ctas = min(64, max(1, -(-M // 256)))
    with _Range("md_ce_tp"):
        nat.check(nat.lib().md_ce_tp(ctypes.byref(prm), ctas, ctypes.c_void_p(nat.stream_ptr(None))), "md_ce_tp")
    n = 3 * M * 4
    comm.comm_stats.add("all_gather", n * c.world, int((c.world - 1) * n))
    return lse, loss
