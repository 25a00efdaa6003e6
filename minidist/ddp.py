"""Data parallelism: gradients averaged in ~25 MB buckets, launched during backward.

Buckets are built over the parameters in *reverse* registration order, which
is roughly the order backward produces their gradients, so bucket 0 fills
first.  A bucket is launched as soon as it is full **and** every lower-numbered
bucket has been launched.  Readiness triggers launches (that is the overlap);
the in-order rule makes the sequence of collectives identical on every rank,
which NCCL needs because it matches collectives by call order (reference
ddp.py:1-35, 234-241).  A callback queued on the autograd engine flushes and
waits at the end of backward, so ``loss.backward(); opt.step()`` is correct
without an explicit sync call (reference ddp.py:201-232).

B200 design.  Each bucket is one contiguous fp32 buffer and every parameter's
``.grad`` is a view into it once the first synchronised backward has run, so
there is no pack/unpack copy.  On CUDA with NCCL, when every rank of the group
is on this node, the buffers live in peer-mapped memory
(:mod:`minidist.parallel.symm`) and a bucket is reduced by one fused kernel
(:func:`minidist.parallel.collectives.bucket_allreduce`) that applies the
``1/W`` scale and reduces over NVLink on a side stream, overlapped with the
rest of backward.  Elsewhere (Gloo, CPU, ``MINIDIST_DDP_REDUCER=nccl``) the
bucket is pre-scaled and handed to ``torch.distributed.all_reduce``.
"""

from __future__ import annotations

import os
import weakref
from collections.abc import Iterator
from contextlib import contextmanager

import torch
import torch.distributed as dist
from torch import nn

from . import comm
from .ops import grads as gradsink

__all__ = ["DistributedDataParallel", "DDP", "wait_all_deferred"]

_DEFAULT_BUCKET_CAP_MB = 25.0
_ALIGN = 64  # elements; keeps every parameter's slice 256-byte aligned for the kernels


class _Bucket:
    """A contiguous run of parameters whose gradients share one flat buffer."""

    def __init__(self, index: int, params: list[nn.Parameter]):
        self.index = index
        self.params = params
        self.offsets: list[int] = []
        off = 0
        for p in params:
            self.offsets.append(off)
            off += (p.numel() + _ALIGN - 1) // _ALIGN * _ALIGN
        self.numel = off  # padded length of the flat buffer
        self.payload_numel = sum(p.numel() for p in params)
        self.buffer: torch.Tensor | None = None
        self.pending = len(params)
        self.work = None
        self.launched = False

    def view_of(self, i: int) -> torch.Tensor:
        p = self.params[i]
        return self.buffer[self.offsets[i] : self.offsets[i] + p.numel()].view_as(p)

    def reset(self) -> None:
        self.pending = len(self.params)
        self.work = None
        self.launched = False


class DistributedDataParallel(nn.Module):
    """Replicate ``module`` over ``process_group`` and average gradients in buckets.

    Parameters match the reference (ddp.py:104-156): ``bucket_cap_mb`` (25),
    ``broadcast_parameters`` (copy rank ``src``'s parameters and buffers at
    construction), ``overlap_with_backward`` (``False`` reduces everything
    after backward, for measuring what overlap is worth).
    """

    def __init__(
        self,
        module: nn.Module,
        process_group: dist.ProcessGroup | None = None,
        bucket_cap_mb: float = _DEFAULT_BUCKET_CAP_MB,
        broadcast_parameters: bool = True,
        overlap_with_backward: bool = True,
        src: int = 0,
        defer_last_buckets: int = 0,
    ):
        """``defer_last_buckets = k``: backward returns without waiting for the all-reduce
        of the last ``k`` buckets.  Their parameters carry the reduction's handle (a CUDA
        event on the peer-memory reducer, a ``Work`` on NCCL / Gloo) as ``_md_grad_event``;
        :class:`minidist.optim.FusedAdamW` updates every other parameter first and waits on
        the handles only for those, so the all-reduce of the gradients produced last in
        backward (the token embedding) overlaps the optimizer.

        Nothing else can see an un-reduced gradient: any other optimizer's ``step`` (a
        global step pre-hook), :meth:`DistributedGradScaler.unscale_
        <minidist.amp.DistributedGradScaler.unscale_>`, the next forward and ``no_sync``
        all wait first.  Code that reads ``.grad`` directly between backward and the
        optimizer step (e.g. ``clip_grad_norm_``) calls :meth:`wait_gradients` or
        :func:`wait_all_deferred` before it."""
        super().__init__()
        self.defer_last_buckets = int(defer_last_buckets)
        self._deferred: list = []
        if self.defer_last_buckets > 0:
            _install_step_guard()
        comm.check_same_layout(list(module.parameters()), process_group, "DistributedDataParallel")
        self.module = module
        self.process_group = process_group
        self.world_size = comm.get_world_size(process_group)
        self.overlap_with_backward = overlap_with_backward
        self.require_backward_grad_sync = True

        if broadcast_parameters and self.world_size > 1:
            self._sync_module_states(src)

        params = [p for p in module.parameters() if p.requires_grad]
        self._buckets = self._build_buckets(params, bucket_cap_mb)
        self._bucket_of: dict[int, tuple[_Bucket, int]] = {
            id(p): (b, i) for b in self._buckets for i, p in enumerate(b.params)
        }
        self._next_to_launch = 0
        self._callback_queued = False
        # Parameters already counted in this backward: a parameter whose
        # gradient a fused kernel wrote reports through ops/grads.py, and
        # autograd may still run its post-accumulate hook afterwards.
        self._ready: set[int] = set()
        self._handles: list = []
        self._reducer = None
        if self.world_size > 1:
            self._reducer = _make_reducer(self)
            self._allocate_buffers()
            self._register_hooks()

    # -- construction -----------------------------------------------------------

    def _sync_module_states(self, src: int) -> None:
        gsrc = src if self.process_group is None else dist.get_global_rank(self.process_group, src)
        with torch.no_grad():
            for p in self.module.parameters():
                comm.broadcast(p.data, src=gsrc, group=self.process_group)
            for b in self.module.buffers():
                if b.is_floating_point() or b.dtype in (torch.int64, torch.int32, torch.bool):
                    comm.broadcast(b.data, src=gsrc, group=self.process_group)

    @staticmethod
    def _build_buckets(params: list[nn.Parameter], cap_mb: float) -> list[_Bucket]:
        cap = int(cap_mb * 1024 * 1024)
        buckets: list[_Bucket] = []
        cur: list[nn.Parameter] = []
        cur_bytes = 0
        for p in reversed(params):
            nbytes = p.numel() * p.element_size()
            if cur and cur_bytes + nbytes > cap:
                buckets.append(_Bucket(len(buckets), cur))
                cur, cur_bytes = [], 0
            cur.append(p)
            cur_bytes += nbytes
        if cur:
            buckets.append(_Bucket(len(buckets), cur))
        return buckets

    def _allocate_buffers(self) -> None:
        total = sum(b.numel for b in self._buckets)
        p0 = self._buckets[0].params[0]
        flat = self._reducer.allocate(total, p0.dtype, p0.device)
        off = 0
        for b in self._buckets:
            b.buffer = flat[off : off + b.numel]
            off += b.numel
            for i, p in enumerate(b.params):
                # Fused kernels write straight into these views (see ops/grads.py).
                gradsink.set_main_grad(p, b.view_of(i))

    def _register_hooks(self) -> None:
        for b in self._buckets:
            for p in b.params:
                self._handles.append(p.register_post_accumulate_grad_hook(self._on_grad_ready))
                self._handles.append(gradsink.add_ready_hook(p, self._on_grad_ready))

    # -- backward-time machinery ------------------------------------------------------

    def _on_grad_ready(self, param: torch.Tensor) -> None:
        if not self.require_backward_grad_sync:
            return
        if id(param) in self._ready:
            return
        self._ready.add(id(param))
        if not self._callback_queued:
            self._callback_queued = True
            try:
                torch.autograd.Variable._execution_engine.queue_callback(self._finalize_backward)
            except Exception:  # pragma: no cover - only legal inside backward
                self._callback_queued = False
        bucket, _ = self._bucket_of[id(param)]
        bucket.pending -= 1
        if self.overlap_with_backward:
            self._launch_ready_buckets()

    def _launch_ready_buckets(self) -> None:
        while self._next_to_launch < len(self._buckets):
            b = self._buckets[self._next_to_launch]
            if b.pending > 0:
                break
            self._launch(b)
            self._next_to_launch += 1

    def _gather(self, b: _Bucket) -> None:
        """Make ``b.buffer`` hold every gradient of the bucket (usually a no-op: grads are views)."""
        for i, p in enumerate(b.params):
            view = b.view_of(i)
            g = p.grad
            if g is None:
                view.zero_()
            elif g.data_ptr() != view.data_ptr():
                view.copy_(g.detach().view_as(view))
            p.grad = view

    def _launch(self, b: _Bucket) -> None:
        self._gather(b)
        self._reducer.launch(b)
        b.launched = True

    def _finalize_backward(self) -> None:
        self._callback_queued = False
        self.finish_gradient_sync()

    def finish_gradient_sync(self) -> None:
        """Launch any bucket not yet launched (in index order) and wait for all of them."""
        if self.world_size == 1 or not self.require_backward_grad_sync:
            return
        while self._next_to_launch < len(self._buckets):
            self._launch(self._buckets[self._next_to_launch])
            self._next_to_launch += 1
        tail = {id(b) for b in self._buckets[len(self._buckets) - self.defer_last_buckets:]} \
            if self.defer_last_buckets > 0 else set()
        self.wait_gradients()  # a previous step's deferred buckets, if nobody consumed them
        for b in self._buckets:
            if b.launched:
                if id(b) in tail and b.work is not None:
                    for p in b.params:
                        p._md_grad_event = b.work
                    self._deferred.extend(b.params)
                else:
                    self._reducer.wait(b)
            b.reset()
        if self._deferred:
            _PENDING.add(self)
        self._next_to_launch = 0
        self._ready.clear()

    # -- public API --------------------------------------------------------------

    def wait_gradients(self) -> None:
        """Order the current stream (or the host, for a ``Work``) after the deferred buckets'
        all-reduce (see ``defer_last_buckets``); a no-op when nothing is pending."""
        if not self._deferred:
            return
        seen: set[int] = set()
        for p in self._deferred:
            h = getattr(p, "_md_grad_event", None)
            if h is not None:
                if id(h) not in seen:
                    seen.add(id(h))
                    wait_handle(h)
                p._md_grad_event = None
        self._deferred = []
        _PENDING.discard(self)

    @contextmanager
    def no_sync(self) -> Iterator[None]:
        """Accumulate gradients locally; the next synchronised backward reduces the sum."""
        self.wait_gradients()
        prev = self.require_backward_grad_sync
        self.require_backward_grad_sync = False
        try:
            yield
        finally:
            self.require_backward_grad_sync = prev

    def forward(self, *args, **kwargs):
        self.wait_gradients()
        return self.module(*args, **kwargs)

    def bucket_summary(self) -> list[tuple[int, int, float]]:
        """``(index, n_params, MB)`` per bucket."""
        return [(b.index, len(b.params), sum(p.numel() * p.element_size() for p in b.params) / 1024**2)
                for b in self._buckets]

    @property
    def reducer_name(self) -> str:
        return "none" if self._reducer is None else self._reducer.name

    def __getattr__(self, name: str):
        try:
            return super().__getattr__(name)
        except AttributeError:
            return getattr(self.module, name)


DDP = DistributedDataParallel


# ---------------------------------------------------------------------------
# Deferred gradients: nobody but an optimizer that asks for them sees them early
# ---------------------------------------------------------------------------

# DDP instances whose last backward left deferred buckets in flight.
_PENDING: weakref.WeakSet = weakref.WeakSet()
_GUARD = None


def wait_handle(h) -> None:
    """Wait for one gradient-reduction handle: a CUDA event (the current stream waits) or a
    ``torch.distributed`` ``Work``."""
    if isinstance(h, torch.cuda.Event):
        torch.cuda.current_stream().wait_event(h)
    else:
        h.wait()


def wait_all_deferred() -> None:
    """Wait for every DDP module's deferred gradient buckets (see ``defer_last_buckets``)."""
    for ddp in list(_PENDING):
        ddp.wait_gradients()


def _step_guard(optimizer, args, kwargs) -> None:
    # An optimizer that orders itself after each parameter's handle (FusedAdamW) declares it;
    # every other optimizer sees fully reduced gradients.
    if _PENDING and not getattr(optimizer, "honours_grad_events", False):
        wait_all_deferred()


def _install_step_guard() -> None:
    global _GUARD
    if _GUARD is None:
        from torch.optim.optimizer import register_optimizer_step_pre_hook

        _GUARD = register_optimizer_step_pre_hook(_step_guard)


# ---------------------------------------------------------------------------
# Reducers
# ---------------------------------------------------------------------------


class _CollectiveReducer:
    """Pre-scale by 1/W, then an async ``all_reduce`` through torch.distributed."""

    name = "nccl"

    def __init__(self, ddp: DistributedDataParallel):
        self.group = ddp.process_group
        self.world = ddp.world_size

    def allocate(self, numel: int, dtype, device) -> torch.Tensor:
        return torch.zeros(numel, dtype=dtype, device=device)

    def launch(self, b: _Bucket) -> None:
        b.buffer.mul_(1.0 / self.world)
        b.work = comm.all_reduce(b.buffer, group=self.group, async_op=True)

    def wait(self, b: _Bucket) -> None:
        if b.work is not None:
            b.work.wait()


def _make_reducer(ddp: DistributedDataParallel):
    choice = os.environ.get("MINIDIST_DDP_REDUCER", "auto")
    p0 = next((p for p in ddp.module.parameters() if p.requires_grad), None)
    if choice != "nccl" and p0 is not None and p0.is_cuda:
        from .parallel import collectives

        r = collectives.make_bucket_reducer(ddp, required=(choice == "fused"))
        if r is not None:
            return r
    return _CollectiveReducer(ddp)
