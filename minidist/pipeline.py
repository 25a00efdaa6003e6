r"""Pipeline (inter-layer) parallelism: GPipe and 1F1B schedules over point-to-point sends.

A stage owns a contiguous slice of layers; activations flow to the next stage
and gradients flow back.  With ``P`` stages and ``M`` microbatches both GPipe
and (non-interleaved) 1F1B idle for the same fill and drain, so both have the
bubble fraction ``(P-1)/(M+P-1)``; 1F1B differs in holding at most ``P - p``
microbatches of activations on stage ``p`` instead of ``M`` (reference
pipeline.py:1-55).

Transport.  Activations and gradients travel as NCCL ``isend``/``irecv``
(Gloo on CPU).  The first message of each kind ("act", "grad") carries a
10-int64 header ``[ndim, d0..d7, dtype_index]`` so the receiver can allocate;
both sides cache it per kind and per direction (reference pipeline.py:77-78,
170-231).  On CUDA, sends and receives are asynchronous to the host: NCCL's
``wait`` only orders the compute stream after the transfer, so the host keeps
queueing work while activations are in flight.

Timeline.  :class:`StageTimeline` records forward/backward/send/recv spans.
On CUDA the spans are CUDA events on the compute stream, so the reported busy
time and bubble are *device* time rather than host enqueue time.
"""

from __future__ import annotations

import time
from collections.abc import Callable, Sequence
from contextlib import contextmanager
from dataclasses import dataclass, field

import torch
import torch.distributed as dist
from torch import nn

from .mesh import ParallelMesh

__all__ = [
    "PipelineStage",
    "GPipeSchedule",
    "OneForwardOneBackwardSchedule",
    "build_schedule",
    "partition_layers",
    "StageTimeline",
    "theoretical_bubble_fraction",
]

_DTYPES = [torch.float32, torch.float16, torch.bfloat16, torch.float64]
_HEADER_LEN = 10


def theoretical_bubble_fraction(num_stages: int, num_microbatches: int) -> float:
    """``(P-1)/(M+P-1)``, the idle fraction of GPipe and non-interleaved 1F1B."""
    if num_stages <= 1:
        return 0.0
    return (num_stages - 1) / (num_microbatches + num_stages - 1)


def partition_layers(layers: Sequence[nn.Module], num_stages: int, stage: int) -> list[nn.Module]:
    """Contiguous near-even split: the first ``len % P`` stages get one extra layer."""
    n = len(layers)
    if num_stages > n:
        raise ValueError(f"{num_stages} stages requested for only {n} layers")
    q, r = divmod(n, num_stages)
    bounds = [0]
    for s in range(num_stages):
        bounds.append(bounds[-1] + q + (1 if s < r else 0))
    return list(layers[bounds[stage] : bounds[stage + 1]])


# ---------------------------------------------------------------------------
# Timeline
# ---------------------------------------------------------------------------


@dataclass
class StageTimeline:
    """Spans ``(kind, microbatch, begin_s, end_s)`` relative to :meth:`start`."""

    events: list[tuple[str, int, float, float]] = field(default_factory=list)
    t0: float = 0.0
    t_end: float = 0.0
    use_cuda_events: bool = False
    _pending: list = field(default_factory=list)
    _ev0: object = None
    _ev_end: object = None

    def start(self) -> None:
        self.events.clear()
        self._pending.clear()
        if self.use_cuda_events:
            self._ev0 = torch.cuda.Event(enable_timing=True)
            self._ev0.record()
        self.t0 = time.perf_counter()

    def stop(self) -> None:
        if self.use_cuda_events:
            self._ev_end = torch.cuda.Event(enable_timing=True)
            self._ev_end.record()
        self.t_end = time.perf_counter()

    def record(self, kind: str, microbatch: int, begin: float, end: float) -> None:
        """Add a host-clock span (``begin``/``end`` from ``time.perf_counter``)."""
        self.events.append((kind, microbatch, begin - self.t0, end - self.t0))

    @contextmanager
    def span(self, kind: str, microbatch: int):
        if self.use_cuda_events:
            b = torch.cuda.Event(enable_timing=True)
            e = torch.cuda.Event(enable_timing=True)
            b.record()
            yield
            e.record()
            self._pending.append((kind, microbatch, b, e))
        else:
            b = time.perf_counter()
            yield
            self.record(kind, microbatch, b, time.perf_counter())

    def _resolve(self) -> None:
        if not self._pending or self._ev0 is None:
            return
        self._ev_end.synchronize()
        for kind, mb, b, e in self._pending:
            self.events.append((kind, mb, self._ev0.elapsed_time(b) / 1e3, self._ev0.elapsed_time(e) / 1e3))
        self._pending.clear()
        self.t_end = self.t0 + self._ev0.elapsed_time(self._ev_end) / 1e3

    @property
    def wall_time(self) -> float:
        self._resolve()
        return self.t_end - self.t0

    def busy_time(self, kinds: tuple[str, ...] = ("forward", "backward")) -> float:
        self._resolve()
        return sum(e - b for k, _, b, e in self.events if k in kinds)

    def comm_time(self) -> float:
        return self.busy_time(("send", "recv"))

    def bubble_fraction(self) -> float:
        """Share of wall time spent outside forward/backward (waiting in recv counts as bubble)."""
        wall = self.wall_time
        if wall <= 0:
            return 0.0
        return max(0.0, 1.0 - self.busy_time() / wall)

    def ascii_gantt(self, width: int = 72) -> str:
        wall = self.wall_time
        if wall <= 0:
            return ""
        row = ["."] * width
        glyph = {"forward": "F", "backward": "B", "send": ">", "recv": "<"}
        for kind, _, b, e in self.events:
            lo = int(b / wall * (width - 1))
            hi = max(lo, int(e / wall * (width - 1)))
            for i in range(lo, min(hi + 1, width)):
                if kind in ("forward", "backward") or row[i] == ".":
                    row[i] = glyph[kind]
        return "".join(row)


# ---------------------------------------------------------------------------
# Point-to-point transport
# ---------------------------------------------------------------------------


class _P2P:
    """Self-describing sends/receives between neighbouring stages.

    Activations travel on the pipeline group and gradients on a second group
    over the same ranks (``ParallelMesh.pp_grad_group``): with NCCL each
    communicator has its own stream, so the two directions cannot block each
    other (one shared stream put the send of activation i+1 in front of the
    receive of gradient i on the first stage, tripling the measured bubble).

    Outgoing and incoming header caches are separate: a middle stage receives
    "act" from its predecessor and sends "act" to its successor, and a shared
    cache would let the incoming header count as already sent.
    """

    def __init__(self, group, device: torch.device, grad_group=None):
        self.group = group
        self.grad_group = grad_group if grad_group is not None else group
        self.device = device
        self._sent: dict[str, tuple[torch.Size, torch.dtype]] = {}
        self._recvd: dict[str, tuple[torch.Size, torch.dtype]] = {}
        self._inflight: list[tuple[object, torch.Tensor]] = []

    def _header(self, t: torch.Tensor) -> torch.Tensor:
        if t.dim() > _HEADER_LEN - 2:
            raise ValueError(f"pipeline tensors may have at most {_HEADER_LEN - 2} dims")
        vals = [t.dim(), *t.shape] + [0] * (_HEADER_LEN - 2 - t.dim()) + [_DTYPES.index(t.dtype)]
        return torch.tensor(vals, dtype=torch.int64, device=self.device)

    def _group_for(self, key: str):
        return self.grad_group if key == "grad" else self.group

    def send(self, tensor: torch.Tensor, dst: int, key: str) -> None:
        tensor = tensor.detach().contiguous()
        grp = self._group_for(key)
        if key not in self._sent:
            hdr = self._header(tensor)
            self._inflight.append((dist.isend(hdr, dst=dst, group=grp), hdr))
            self._sent[key] = (tensor.shape, tensor.dtype)
        self._inflight.append((dist.isend(tensor, dst=dst, group=grp), tensor))

    def recv(self, src: int, key: str) -> torch.Tensor:
        grp = self._group_for(key)
        if key not in self._recvd:
            hdr = torch.zeros(_HEADER_LEN, dtype=torch.int64, device=self.device)
            dist.recv(hdr, src=src, group=grp)
            vals = hdr.tolist()
            self._recvd[key] = (torch.Size(vals[1 : 1 + vals[0]]), _DTYPES[vals[-1]])
        shape, dtype = self._recvd[key]
        buf = torch.empty(shape, dtype=dtype, device=self.device)
        work = dist.irecv(buf, src=src, group=grp)
        work.wait()
        return buf

    def drain(self) -> None:
        for work, _ in self._inflight:
            work.wait()
        self._inflight.clear()


# ---------------------------------------------------------------------------
# Stage and schedules
# ---------------------------------------------------------------------------


class PipelineStage(nn.Module):
    """This rank's layers; the last stage also owns ``loss_fn(output, target)``."""

    def __init__(self, module: nn.Module, mesh: ParallelMesh,
                 loss_fn: Callable[[torch.Tensor, torch.Tensor], torch.Tensor] | None = None):
        super().__init__()
        self.module = module
        self.mesh = mesh
        self.loss_fn = loss_fn
        if mesh.is_last_stage and loss_fn is None:
            raise ValueError("the last pipeline stage needs a loss_fn")

    def forward(self, x):
        return self.module(x)


class _Schedule:
    name = "base"

    def __init__(self, stage: PipelineStage, mesh: ParallelMesh, num_microbatches: int):
        if num_microbatches < 1:
            raise ValueError("num_microbatches must be >= 1")
        self.stage, self.mesh, self.num_microbatches = stage, mesh, num_microbatches
        self.timeline = StageTimeline(use_cuda_events=mesh.device.type == "cuda")
        self.max_activations_in_flight = 0
        self.loss_scale = 1.0  # fp16 loss scaling must be applied before backward
        self._p2p = _P2P(mesh.pp_group, mesh.device, getattr(mesh, "pp_grad_group", None))
        self._live: list[tuple[torch.Tensor | None, torch.Tensor]] = []
        self._losses: list[torch.Tensor] = []

    # -- one microbatch --------------------------------------------------------

    def _forward(self, i: int, inputs, targets) -> None:
        mesh, tl = self.mesh, self.timeline
        if mesh.is_first_stage:
            x = inputs[i]
        else:
            with tl.span("recv", i):
                x = self._p2p.recv(mesh.prev_stage_rank, "act")
            x.requires_grad_(True)
        with tl.span("forward", i):
            y = self.stage(x)
            if mesh.is_last_stage:
                # 1/M makes the accumulated gradient the gradient of the batch mean.
                loss = self.stage.loss_fn(y, targets[i]) / self.num_microbatches
                self._losses.append(loss.detach())
                y = loss * self.loss_scale if self.loss_scale != 1.0 else loss
        if not mesh.is_last_stage:
            with tl.span("send", i):
                self._p2p.send(y, mesh.next_stage_rank, "act")
        self._live.append((None if mesh.is_first_stage else x, y))
        self.max_activations_in_flight = max(self.max_activations_in_flight, len(self._live))

    def _backward(self, i: int) -> None:
        mesh, tl = self.mesh, self.timeline
        x, y = self._live.pop(0)
        if mesh.is_last_stage:
            with tl.span("backward", i):
                torch.autograd.backward(y)
        else:
            with tl.span("recv", i):
                g = self._p2p.recv(mesh.next_stage_rank, "grad")
            with tl.span("backward", i):
                torch.autograd.backward(y, grad_tensors=g)
        if not mesh.is_first_stage:
            assert x is not None and x.grad is not None, "stage input received no gradient"
            with tl.span("send", i):
                self._p2p.send(x.grad, mesh.prev_stage_rank, "grad")

    def _split(self, batch):
        if batch is None:
            return None
        if batch.size(0) % self.num_microbatches:
            raise ValueError(f"batch of {batch.size(0)} is not divisible by {self.num_microbatches} microbatches")
        return list(batch.chunk(self.num_microbatches, dim=0))

    def _order(self) -> list[tuple[str, int]]:
        raise NotImplementedError

    def step(self, inputs=None, targets=None):
        """Run every microbatch's forward and backward; return the summed (1/M-scaled) loss on the last stage."""
        mb_in, mb_tg = self._split(inputs), self._split(targets)
        self.timeline.start()
        self._live.clear()
        self._losses.clear()
        self.max_activations_in_flight = 0
        for op, i in self._order():
            if op == "F":
                self._forward(i, mb_in, mb_tg)
            else:
                self._backward(i)
        self._p2p.drain()
        self.timeline.stop()
        return torch.stack(self._losses).sum() if self._losses else None

    def report(self) -> dict[str, float]:
        tl = self.timeline
        return {
            "wall_s": tl.wall_time,
            "busy_s": tl.busy_time(),
            "comm_s": tl.comm_time(),
            "measured_bubble": tl.bubble_fraction(),
            "theoretical_bubble": theoretical_bubble_fraction(self.mesh.pp_size, self.num_microbatches),
            "peak_activations_in_flight": float(self.max_activations_in_flight),
        }


class GPipeSchedule(_Schedule):
    """All forwards, then all backwards: peak activations grow with ``M``."""

    name = "gpipe"

    def _order(self):
        M = self.num_microbatches
        return [("F", i) for i in range(M)] + [("B", i) for i in range(M)]


class OneForwardOneBackwardSchedule(_Schedule):
    """1F1B: ``P-1-p`` warm-up forwards, then alternate F/B, then drain the backwards."""

    name = "1f1b"

    def _order(self):
        M, P, p = self.num_microbatches, self.mesh.pp_size, self.mesh.pp_rank
        warm = min(P - 1 - p, M)
        order = [("F", i) for i in range(warm)]
        for k in range(M - warm):
            order += [("F", warm + k), ("B", k)]
        order += [("B", i) for i in range(M - warm, M)]
        return order


_SCHEDULES = {"gpipe": GPipeSchedule, "1f1b": OneForwardOneBackwardSchedule}


def build_schedule(name: str, stage: PipelineStage, mesh: ParallelMesh, num_microbatches: int) -> _Schedule:
    if name not in _SCHEDULES:
        raise ValueError(f"unknown schedule {name!r}; choose from {sorted(_SCHEDULES)}")
    return _SCHEDULES[name](stage, mesh, num_microbatches)
