"""Process bootstrap and the framework's single door to ``torch.distributed``.

Everything above this module (mesh, DDP, FSDP, tensor/pipeline parallelism,
AMP) reaches collectives through the wrappers here, for two reasons that match
``minidist/comm.py`` of the reference (comm.py:1-13):

* device and backend selection happen in exactly one place;
* every collective is byte-counted, so benchmarks can print *measured* traffic
  beside the analytic prediction.  Our fused NVLink kernels
  (:mod:`minidist.parallel.collectives`) report through the same
  :data:`comm_stats` object with the same bus-byte formulas, so a run that
  switches from NCCL to the fused kernels keeps comparable numbers.

Bus bytes for an ``N``-byte payload over ``W`` ranks (ring accounting, the
convention ``nccl-tests`` uses): all-reduce ``2(W-1)/W*N``, all-gather
``(W-1)/W*N_out``, reduce-scatter ``(W-1)/W*N_in``, broadcast ``N``
(reference comm.py:57-100).
"""

from __future__ import annotations

import os
import socket
from collections.abc import Iterator
from contextlib import contextmanager
from dataclasses import dataclass, field
from datetime import timedelta

import torch
import torch.distributed as dist

__all__ = [
    "CommStats",
    "comm_stats",
    "record_comm",
    "init_distributed",
    "shutdown_distributed",
    "is_distributed",
    "get_rank",
    "get_world_size",
    "is_primary",
    "barrier",
    "all_reduce",
    "all_gather_into_tensor",
    "reduce_scatter_tensor",
    "broadcast",
    "print_rank0",
    "current_device",
    "bus_bytes",
]


# ---------------------------------------------------------------------------
# Byte accounting
# ---------------------------------------------------------------------------


def bus_bytes(op: str, payload: int, world: int) -> int:
    """Bytes that cross the interconnect for ``op`` on a ``payload``-byte buffer."""
    if world <= 1:
        return 0
    frac = (world - 1) / world
    if op == "all_reduce":
        return int(2 * frac * payload)
    if op in ("all_gather", "reduce_scatter"):
        return int(frac * payload)
    if op == "broadcast":
        return int(payload)
    raise ValueError(f"unknown collective {op!r}")


@dataclass
class _OpStat:
    count: int = 0
    payload_bytes: int = 0
    bus_bytes: int = 0


@dataclass
class CommStats:
    """Per-collective counters: number of calls, caller payload bytes, bus bytes.

    Disabled by default (the add is a single branch); :func:`record_comm` turns
    it on for a block.
    """

    enabled: bool = False
    ops: dict[str, _OpStat] = field(default_factory=dict)

    def add(self, op: str, payload_bytes: int, bus: int) -> None:
        if not self.enabled:
            return
        s = self.ops.get(op)
        if s is None:
            s = self.ops[op] = _OpStat()
        s.count += 1
        s.payload_bytes += int(payload_bytes)
        s.bus_bytes += int(bus)

    def reset(self) -> None:
        self.ops.clear()

    def total_bus_bytes(self) -> int:
        return sum(s.bus_bytes for s in self.ops.values())

    def as_rows(self) -> list[tuple[str, int, int, int]]:
        return sorted((k, s.count, s.payload_bytes, s.bus_bytes) for k, s in self.ops.items())


comm_stats = CommStats()


@contextmanager
def record_comm() -> Iterator[CommStats]:
    """Count collective traffic inside the block (counters are reset on entry)."""
    prev = comm_stats.enabled
    comm_stats.enabled = True
    comm_stats.reset()
    try:
        yield comm_stats
    finally:
        comm_stats.enabled = prev


# ---------------------------------------------------------------------------
# Bootstrap
# ---------------------------------------------------------------------------


def _default_backend() -> str:
    return "nccl" if (torch.cuda.is_available() and dist.is_nccl_available()) else "gloo"


def _free_port() -> int:
    with socket.socket(socket.AF_INET, socket.SOCK_STREAM) as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def init_distributed(backend: str | None = None, timeout_seconds: int = 1800) -> tuple[int, int, torch.device]:
    """Create the default process group from torchrun's environment.

    Returns ``(rank, world_size, device)``.  Without torchrun it makes a
    one-rank world, so every script also runs as a plain ``python`` command
    (reference comm.py:129-164).  Under NCCL the process is bound to
    ``cuda:LOCAL_RANK`` *before* the group exists, because NCCL derives its
    topology from the current device.
    """
    if dist.is_available() and dist.is_initialized():
        return get_rank(), get_world_size(), current_device()

    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    backend = backend or _default_backend()
    if backend == "nccl":
        if not torch.cuda.is_available():
            raise RuntimeError("backend='nccl' requested but no CUDA device is visible")
        torch.cuda.set_device(local_rank)

    os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
    if world == 1 and "MASTER_PORT" not in os.environ:
        # A lone process must not collide with another run on the default port.
        os.environ["MASTER_PORT"] = str(_free_port())
    os.environ.setdefault("MASTER_PORT", "29500")

    kwargs = {}
    if backend == "nccl":
        kwargs["device_id"] = torch.device("cuda", local_rank)
    dist.init_process_group(
        backend=backend,
        rank=rank,
        world_size=world,
        timeout=timedelta(seconds=timeout_seconds),
        **kwargs,
    )
    return rank, world, current_device()


def shutdown_distributed() -> None:
    """Release native communicators, then barrier and destroy the process group."""
    if not (dist.is_available() and dist.is_initialized()):
        return
    try:
        from .parallel import symm

        symm.release_all()
    except Exception:  # pragma: no cover - best effort on teardown
        pass
    dist.barrier()
    dist.destroy_process_group()


def current_device() -> torch.device:
    if torch.cuda.is_available():
        return torch.device("cuda", torch.cuda.current_device())
    return torch.device("cpu")


def is_distributed() -> bool:
    return dist.is_available() and dist.is_initialized()


def get_rank(group: dist.ProcessGroup | None = None) -> int:
    return dist.get_rank(group) if is_distributed() else 0


def get_world_size(group: dist.ProcessGroup | None = None) -> int:
    return dist.get_world_size(group) if is_distributed() else 1


def is_primary() -> bool:
    return get_rank() == 0


def barrier(group: dist.ProcessGroup | None = None) -> None:
    if is_distributed():
        dist.barrier(group)


def print_rank0(*args, **kwargs) -> None:
    if is_primary():
        kwargs.setdefault("flush", True)
        print(*args, **kwargs)


# ---------------------------------------------------------------------------
# Instrumented collectives (NCCL / Gloo).  Size-1 groups short-circuit.
# ---------------------------------------------------------------------------


def _nbytes(t: torch.Tensor) -> int:
    return t.numel() * t.element_size()


def all_reduce(tensor, op=dist.ReduceOp.SUM, group=None, async_op: bool = False):
    world = get_world_size(group)
    if world == 1:
        return None
    n = _nbytes(tensor)
    comm_stats.add("all_reduce", n, bus_bytes("all_reduce", n, world))
    return dist.all_reduce(tensor, op=op, group=group, async_op=async_op)


def all_gather_into_tensor(output, input_, group=None, async_op: bool = False):
    world = get_world_size(group)
    if world == 1:
        output.copy_(input_)
        return None
    n = _nbytes(output)
    comm_stats.add("all_gather", n, bus_bytes("all_gather", n, world))
    return dist.all_gather_into_tensor(output, input_, group=group, async_op=async_op)


def reduce_scatter_tensor(output, input_, op=dist.ReduceOp.SUM, group=None, async_op: bool = False):
    world = get_world_size(group)
    if world == 1:
        output.copy_(input_)
        return None
    n = _nbytes(input_)
    comm_stats.add("reduce_scatter", n, bus_bytes("reduce_scatter", n, world))
    return dist.reduce_scatter_tensor(output, input_, op=op, group=group, async_op=async_op)


def broadcast(tensor, src: int, group=None, async_op: bool = False):
    if get_world_size(group) == 1:
        return None
    n = _nbytes(tensor)
    comm_stats.add("broadcast", n, n)
    return dist.broadcast(tensor, src=src, group=group, async_op=async_op)


def check_same_layout(params, group=None, what: str = "module") -> None:
    """Raise on every rank if the parameter layout (shapes, dtypes, order) differs across ``group``.

    DDP and FSDP call this before their first collective: with mismatched
    layouts the parameter broadcast and the bucket / shard collectives would
    otherwise fail in confusing ways or wait until the process-group timeout.
    One 64-bit digest per rank is all-gathered.
    """
    import hashlib

    if not is_distributed() or get_world_size(group) == 1:
        return
    desc = repr([(tuple(p.shape), str(p.dtype)) for p in params]).encode()
    digest = int.from_bytes(hashlib.sha256(desc).digest()[:8], "little", signed=True)
    dev = current_device() if dist.get_backend(group) == "nccl" else torch.device("cpu")
    mine = torch.tensor([digest], dtype=torch.int64, device=dev)
    out = torch.empty(get_world_size(group), dtype=torch.int64, device=dev)
    dist.all_gather_into_tensor(out, mine, group=group)
    vals = out.tolist()
    if any(v != vals[0] for v in vals):
        bad = [r for r, v in enumerate(vals) if v != vals[0]]
        raise RuntimeError(f"{what}: parameter layout differs across ranks (ranks {bad} differ from rank 0); "
                           "every rank must build the same model")
