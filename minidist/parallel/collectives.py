"""Collectives of the fused B200 path.

* :class:`FusedBucketReducer` — DDP's bucket reducer on peer memory: the
  gradient buckets live in a :class:`~minidist.parallel.symm.SymmBuffer`
  (every parameter's ``.grad`` is a view into it), and each bucket is averaged
  by one ``md_ar_bucket_kernel`` launch (1/W scale + reduce-scatter +
  all-gather over NVLink, csrc/symm.cu) on a side stream, ordered after the
  compute stream with CUDA events.  Launch order is bucket 0, 1, 2, ... on
  every rank, as with NCCL.
* :func:`all_reduce_` / :func:`gemm_all_reduce` — tensor-parallel reductions;
  NCCL for now.

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
        ("epoch", ctypes.c_uint32),
        ("channel", ctypes.c_int),
        ("timeout_ns", ctypes.c_ulonglong),
        ("status", ctypes.c_void_p),
    ]


nat.declare("md_allreduce", "i:pip")


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
    p.epoch = comm_.next_epoch(channel) & 0x7FFFFFFF
    p.channel = channel
    p.timeout_ns = _timeout_ns()
    p.status = nat.status_ptr()
    ctas = lib.md_allreduce_ctas(n, buf.world)
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
# Tensor parallel (NCCL)
# ---------------------------------------------------------------------------


def all_reduce_(t: torch.Tensor, group) -> torch.Tensor:
    comm.all_reduce(t, group=group)
    return t


def gemm_all_reduce(x_local, w_local, bias, resid, group):
    out = G.linear_fwd(x_local, w_local)
    comm.all_reduce(out, group=group)
    acc = out.float()
    if bias is not None:
        acc += bias
    if resid is not None:
        acc += resid.float()
    res = G.empty_padded(out.shape[0], out.shape[1], device=out.device)
    res.copy_(acc)
    return res
