"""Fully sharded data parallelism (ZeRO-3): parameters, gradients and optimizer state sharded.

Per rank, DDP holds ``params + grads + fp32 master + Adam m, v`` for the whole
model; FSDP holds ``1/W`` of each plus one transient unit of gathered
parameters (reference fsdp.py:1-22).  The module is split into *units* (one
per ``unit_types`` match, found by a pre-order walk, plus a root unit for the
leftovers).  Each unit:

* flattens its parameters into one buffer padded to a multiple of ``W`` and
  keeps rank ``r``'s slice ``[r*shard, (r+1)*shard)`` as an fp32 parameter
  (``flat_shard``) — the only thing the optimizer sees;
* points every original parameter's ``.data`` at a view of ``_full``, a
  gathered buffer in ``param_dtype`` whose *storage* is freed between uses
  (``untyped_storage().resize_(0)``) and re-filled by an all-gather, so the
  views survive while the bytes come and go (reference fsdp.py:23-48);
* gathers before forward (and again before backward unless
  ``reshard_after_forward=False``, the ZeRO-2-like mode), and once all its
  parameters have gradients, reduce-scatters them in ``reduce_dtype`` with a
  ``1/W`` pre-scale, accumulates into ``flat_shard.grad`` and frees the full
  gradients.

B200 design.  On CUDA the gather for the *next* unit is issued on a side
stream while the current unit computes (the reference gathers synchronously,
fsdp.py:172-182), so NVLink traffic overlaps compute; the gather and the
reduce-scatter of gradients is one peer-memory kernel (md_rs_shard in
csrc/symm.cu: sum of this rank's shard over every rank's fp32 full gradient,
1/W scale, accumulate into the shard gradient -- or, with ``fused_adamw``, the
AdamW update of the shard) when every rank of the group is on this node; NCCL
otherwise.  On the same path the fp32 shards live in a symmetric buffer and the
gather is md_ag_shards (csrc/symm.cu): one kernel that reads every rank's shard
over NVLink and writes the gathered unit in ``param_dtype`` (the reference's
cast + all-gather, fsdp.py:172-182, as one pass).  A reduce-scatter kernel is
ordered after any gather still in flight, so the two cross-rank kernels never
hold SMs against each other.
"""

from __future__ import annotations

from collections.abc import Iterator, Sequence
from contextlib import contextmanager
from contextlib import nullcontext as _nullctx

import torch
import torch.distributed as dist
from torch import nn

from . import comm
from .ops import grads as gradsink

__all__ = ["FullyShardedDataParallel", "FSDP", "MixedPrecisionPolicy"]


class MixedPrecisionPolicy:
    """``param_dtype`` (gathered parameters), ``reduce_dtype`` (gradient reduce-scatter),
    ``keep_low_precision_shard`` (store the shard in ``param_dtype`` instead of fp32)."""

    def __init__(self, param_dtype: torch.dtype = torch.float32, reduce_dtype: torch.dtype = torch.float32,
                 keep_low_precision_shard: bool = False):
        self.param_dtype = param_dtype
        self.reduce_dtype = reduce_dtype
        self.keep_low_precision_shard = keep_low_precision_shard

    def __repr__(self) -> str:
        return f"MixedPrecisionPolicy(param={self.param_dtype}, reduce={self.reduce_dtype})"


class _FSDPUnit:
    def __init__(self, module: nn.Module, params: list[nn.Parameter], group, policy: MixedPrecisionPolicy,
                 reshard_after_forward: bool, device: torch.device, name: str, align: int = 1):
        self.module, self.params, self.group, self.policy = module, params, group, policy
        self.reshard_after_forward = reshard_after_forward
        self.name = name
        self.world = comm.get_world_size(group)
        self.rank = comm.get_rank(group)
        self.shapes = [p.shape for p in params]
        self.numels = [p.numel() for p in params]
        self.total_numel = sum(self.numels)
        self.shard_numel = -(-self.total_numel // self.world)
        self.shard_numel = -(-self.shard_numel // align) * align
        self.padded_numel = self.shard_numel * self.world

        src_dtype = params[0].dtype
        shard_dtype = policy.param_dtype if policy.keep_low_precision_shard else src_dtype
        flat = torch.cat([p.detach().reshape(-1).to(device=device, dtype=src_dtype) for p in params])
        if self.padded_numel > self.total_numel:
            flat = torch.cat([flat, flat.new_zeros(self.padded_numel - self.total_numel)])
        lo = self.rank * self.shard_numel
        self.flat_shard = nn.Parameter(flat[lo : lo + self.shard_numel].clone().to(shard_dtype))
        del flat

        self._full = torch.empty(self.padded_numel, dtype=policy.param_dtype, device=device)
        off = 0
        for p, n, shape in zip(params, self.numels, self.shapes, strict=True):
            p.data = self._full[off : off + n].view(shape)
            off += n
        self._unsharded = True
        self._gather_event = None  # CUDA event of an in-flight prefetch gather
        self.reshard()
        self._pending = 0
        self._grad_acc: torch.Tensor | None = None  # fp32 full grads written by fused kernels
        self._hook_handles: list = []
        # Peer-memory reduce-scatter: (communicator, symmetric buffer, element offset) or None.
        self._peer: tuple | None = None
        # Peer-memory gather: (communicator, symmetric shard buffer, element offset) or None.
        self._peer_shard: tuple | None = None
        self._peer_shard_bf16: tuple | None = None  # bf16 copies of the shards (bf16 gathers)
        self._owner_state: dict | None = None  # shared with the FSDP module: last gather event
        self._adam: dict | None = None  # fused AdamW: hyper-parameters, m, v, step

    # -- gather / free -------------------------------------------------------------

    @property
    def is_unsharded(self) -> bool:
        return self._unsharded

    def _gather_into_full(self) -> None:
        self._full.untyped_storage().resize_(self.padded_numel * self._full.element_size())
        if self._peer_shard is not None:
            from .parallel import collectives

            self._invalidate_casts()
            comm_, buf, off = self._peer_shard
            bf = getattr(self, "_peer_shard_bf16", None)
            if bf is not None:
                from .models import fused_gpt

                shard = self.flat_shard
                if getattr(shard, fused_gpt._SHADOW_VER, None) != shard._version:
                    # The bf16 copy is stale (first gather, or the shard changed outside the
                    # optimizer): refresh it locally before peers read it.
                    getattr(shard, fused_gpt._SHADOW).copy_(shard.detach())
                    setattr(shard, fused_gpt._SHADOW_VER, shard._version)
                comm_, buf, off = bf
                collectives.all_gather_shards(buf, comm_, off, self.shard_numel, self._full, src_bf16=True)
            else:
                collectives.all_gather_shards(buf, comm_, off, self.shard_numel, self._full)
            return
        self._invalidate_casts()
        src = self.flat_shard.detach()
        if src.dtype != self.policy.param_dtype:
            src = src.to(self.policy.param_dtype)
        comm.all_gather_into_tensor(self._full, src.contiguous(), group=self.group)

    def _invalidate_casts(self) -> None:
        """Mark the fused path's cached bf16 casts of this unit's parameters stale.

        A gather rewrites the parameters' bytes (``.data`` views of ``_full``) without touching
        their version counters -- a ``.data`` view keeps its own counter, and bumping it would
        trip autograd's saved-tensor check in the portable path -- so the cast cache is told
        directly."""
        for p in self.params:
            if getattr(p, "_md_bf16_ver", None) is not None:
                p._md_bf16_ver = None

    def unshard(self) -> None:
        if not self._unsharded and self._owner_state is not None:
            # Peer-memory path: every gather runs on the communication stream (see _reduce_scatter_peer).
            self.prefetch(self._owner_state["stream"])
        if self._unsharded:
            if self._gather_event is not None:
                torch.cuda.current_stream().wait_event(self._gather_event)
                self._gather_event = None
            return
        self._gather_into_full()
        self._unsharded = True

    def prefetch(self, stream: torch.cuda.Stream) -> None:
        """Start this unit's gather on ``stream`` (CUDA only)."""
        if self._unsharded:
            return
        stream.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(stream):
            self._gather_into_full()
            ev = torch.cuda.Event()
            ev.record(stream)
        self._full.record_stream(torch.cuda.current_stream())
        self._gather_event = ev
        self._unsharded = True

    def reshard(self) -> None:
        if not self._unsharded:
            return
        if self._gather_event is not None:
            torch.cuda.current_stream().wait_event(self._gather_event)
            self._gather_event = None
        self._full.untyped_storage().resize_(0)
        self._unsharded = False

    # -- gradients -------------------------------------------------------------------

    def arm_gradient_reduction(self) -> None:
        self._pending = sum(1 for p in self.params if p.requires_grad)
        self._ready: set[int] = set()

    def on_param_grad_ready(self, param: torch.Tensor, sync: bool) -> None:
        # Count each parameter once per backward (a fused-kernel gradient may
        # be reported both through ops/grads.py and by autograd's hook).
        ready = getattr(self, "_ready", None)
        if ready is not None:
            if id(param) in ready:
                return
            ready.add(id(param))
        self._pending -= 1
        if self._pending > 0:
            return
        if sync:
            self.reduce_scatter_grads()
        # Always free after backward: a gathered copy kept past the optimizer
        # step would be stale on the next forward (reference fsdp.py:201-213).
        self.reshard()

    def _full_grad_buffer(self) -> torch.Tensor:
        """fp32 buffer for the fused kernels' full gradients (laid out like ``_full``); with the
        peer-memory reduce-scatter it is this unit's slice of the symmetric gradient buffer."""
        if self._grad_acc is None:
            if self._peer is not None:
                _, buf, off = self._peer
                self._grad_acc = buf.view(torch.float32, off * 4, self.padded_numel)
            else:
                self._grad_acc = torch.zeros(self.padded_numel, dtype=self.policy.reduce_dtype,
                                             device=self.flat_shard.device)
            off = 0
            for p, n, shape in zip(self.params, self.numels, self.shapes, strict=True):
                gradsink.set_main_grad(p, self._grad_acc[off : off + n].view(shape))
                off += n
        return self._grad_acc

    def _reduce_scatter_peer(self) -> None:
        """Reduce-scatter through peer memory: the full fp32 gradients sit in this rank's slice of
        the symmetric buffer; one kernel sums this rank's shard over every rank, scales by 1/W and
        accumulates into ``flat_shard.grad`` -- or applies AdamW to the shard in place."""
        from .parallel import collectives

        comm_, buf, off = self._peer
        full = self._full_grad_buffer()
        o = 0
        with torch.no_grad():
            for p, n in zip(self.params, self.numels, strict=True):
                slot = full[o : o + n]
                g = p.grad
                if g is None and getattr(p, "_md_grad_written", False):
                    pass  # a fused kernel wrote the fp32 gradient of a low-precision view in place
                elif g is not None and g.data_ptr() == slot.data_ptr():
                    pass  # written in place (fused kernels' main gradient, or autograd accumulating into it)
                elif g is not None:
                    slot.copy_(g.detach().reshape(-1))
                else:
                    slot.zero_()  # no gradient this step
                o += n
        shard = self.flat_shard
        acc = shard.grad is not None
        if self._adam is None and not acc:
            shard.grad = torch.empty(self.shard_numel, dtype=torch.float32, device=shard.device)
        # The reduce-scatter runs on the module's communication stream, after this unit's
        # gradients on the compute stream; the backward's end makes the compute stream wait
        # for it (FullyShardedDataParallel._end_of_backward).  Gathers and reduce-scatters share
        # that one stream, so the cross-rank kernels of a rank run one at a time, in the same
        # order on every rank.
        stream = self._owner_state["stream"] if self._owner_state is not None else None
        if stream is not None:
            stream.wait_stream(torch.cuda.current_stream())
            if shard.grad is not None:
                shard.grad.record_stream(stream)
        with torch.cuda.stream(stream) if stream is not None else _nullctx():
            if self._adam is not None:
                a = self._adam
                a["step"] += 1
                b1, b2 = a["betas"]
                sh = None
                if self._peer_shard_bf16 is not None:
                    from .models import fused_gpt

                    sh = getattr(shard, fused_gpt._SHADOW, None)
                collectives.reduce_scatter_shard(buf, comm_, off, self.shard_numel, None, False, 1.0 / self.world,
                                                 adam=(shard.data, a["m"], a["v"], a["lr"], b1, b2, a["eps"],
                                                       a["weight_decay"], a["step"]), p_bf16=sh)
                if sh is not None:
                    from .models import fused_gpt

                    setattr(shard, fused_gpt._SHADOW_VER, shard._version)  # updated in the same pass
            else:
                collectives.reduce_scatter_shard(buf, comm_, off, self.shard_numel, shard.grad, acc,
                                                 1.0 / self.world)
        if stream is not None:
            self._owner_state["pending"] = True
        for p in self.params:
            p.grad = None
            p._md_grad_written = False

    def reduce_scatter_grads(self) -> None:
        if self._peer is not None:
            self._reduce_scatter_peer()
            return
        rdt = self.policy.reduce_dtype
        dev = self.flat_shard.device
        buf = torch.zeros(self.padded_numel, dtype=rdt, device=dev)
        off = 0
        for p, n in zip(self.params, self.numels, strict=True):
            g = p.grad
            if g is None and self._grad_acc is not None and getattr(p, "_md_grad_written", False):
                g = gradsink.main_grad(p)
            if g is not None:
                buf[off : off + n].copy_(g.detach().reshape(-1))
            off += n
        if self.world > 1:
            buf.div_(self.world)
            out = torch.empty(self.shard_numel, dtype=rdt, device=dev)
            comm.reduce_scatter_tensor(out, buf, group=self.group)
        else:
            out = buf
        out = out.to(self.flat_shard.dtype)
        if self.flat_shard.grad is None:
            self.flat_shard.grad = out
        else:
            self.flat_shard.grad.add_(out)
        for p in self.params:
            p.grad = None
            p._md_grad_written = False

    def numel_report(self) -> tuple[int, int]:
        return self.total_numel, self.shard_numel


class FullyShardedDataParallel(nn.Module):
    """Shard ``module`` over ``process_group`` (reference fsdp.py:247-501 for the API)."""

    def __init__(
        self,
        module: nn.Module,
        unit_types: Sequence[type] = (),
        process_group: dist.ProcessGroup | None = None,
        mixed_precision: MixedPrecisionPolicy | None = None,
        reshard_after_forward: bool = True,
        reshard_root_after_forward: bool = False,
        broadcast_parameters: bool = True,
        device: torch.device | None = None,
        prefetch: bool = True,
        fused_adamw: dict | None = None,
    ):
        """``fused_adamw`` (dict with ``lr``, ``betas``, ``eps``, ``weight_decay``) applies AdamW to
        each shard inside the gradient reduce-scatter kernel, right when the unit's gradients are
        complete (peer-memory path only; no separate optimizer for these parameters)."""
        super().__init__()
        comm.check_same_layout(list(module.parameters()), process_group, "FullyShardedDataParallel")
        self.module = module
        self.process_group = process_group
        self.world_size = comm.get_world_size(process_group)
        self.policy = mixed_precision or MixedPrecisionPolicy()
        self.require_backward_grad_sync = True
        device = device or comm.current_device()
        if broadcast_parameters and self.world_size > 1:
            gsrc = 0 if process_group is None else dist.get_global_rank(process_group, 0)
            with torch.no_grad():
                for p in module.parameters():
                    comm.broadcast(p.data, src=gsrc, group=process_group)
                for b in module.buffers():
                    comm.broadcast(b.data, src=gsrc, group=process_group)
        self._peer_comm = None
        if device.type == "cuda" and self.world_size > 1 and self.policy.reduce_dtype == torch.float32:
            from .parallel import collectives

            self._peer_comm = collectives.fsdp_communicator(process_group)
        self._align = 8 if self._peer_comm is not None else 1
        self._units = self._build_units(module, tuple(unit_types), reshard_after_forward,
                                        reshard_root_after_forward, device)
        if self._peer_comm is not None:
            total = sum(u.padded_numel for u in self._units)
            self._grad_buf = self._peer_comm.buffer(f"fsdp_grads_{id(self)}", total * 4)
            off = 0
            for u in self._units:
                u._peer = (self._peer_comm, self._grad_buf, off)
                u._full_grad_buffer()  # fused kernels write gradients straight into the symmetric buffer
                off += u.padded_numel
            # One communication stream for every peer-memory gather and reduce-scatter.
            self._gather_state: dict = {"stream": torch.cuda.Stream(device=device), "pending": False}
            if all(u.flat_shard.dtype == torch.float32 and u.policy.param_dtype in (torch.float32, torch.bfloat16)
                   for u in self._units) and collectives.fsdp_gather_enabled():
                # fp32 shards move into a symmetric buffer so peers can read them.
                total_shard = sum(u.shard_numel for u in self._units)
                self._shard_buf = self._peer_comm.buffer(f"fsdp_shards_{id(self)}", total_shard * 4)
                off = 0
                for u in self._units:
                    view = self._shard_buf.view(torch.float32, off * 4, u.shard_numel)
                    view.copy_(u.flat_shard.data)
                    u.flat_shard.data = view
                    u._peer_shard = (self._peer_comm, self._shard_buf, off)
                    u._owner_state = self._gather_state
                    off += u.shard_numel
                if all(u.policy.param_dtype == torch.bfloat16 for u in self._units):
                    # bf16 gathers read a bf16 copy of every fp32 shard, kept next to it in
                    # symmetric memory: the optimizer writes it in the same pass as the update
                    # (FusedAdamW's weight shadow, or the fused AdamW of the reduce-scatter), so
                    # a gather moves half the bytes and casts nothing.
                    from .models import fused_gpt

                    self._shard_bf16_buf = self._peer_comm.buffer(f"fsdp_shards_bf16_{id(self)}", total_shard * 2)
                    off = 0
                    for u in self._units:
                        view = self._shard_bf16_buf.view(torch.bfloat16, off * 2, u.shard_numel)
                        setattr(u.flat_shard, fused_gpt._SHADOW, view)
                        setattr(u.flat_shard, fused_gpt._SHADOW_VER, None)  # filled at the first gather
                        u._peer_shard_bf16 = (self._peer_comm, self._shard_bf16_buf, off)
                        off += u.shard_numel
                torch.cuda.synchronize(device)
        if fused_adamw is not None:
            if self._peer_comm is None or any(u.flat_shard.dtype != torch.float32 for u in self._units):
                raise ValueError("fused_adamw needs the peer-memory reduce-scatter and fp32 shards")
            for u in self._units:
                u._adam = {"lr": float(fused_adamw.get("lr", 1e-3)),
                           "betas": tuple(fused_adamw.get("betas", (0.9, 0.999))),
                           "eps": float(fused_adamw.get("eps", 1e-8)),
                           "weight_decay": float(fused_adamw.get("weight_decay", 0.01)),
                           "m": torch.zeros_like(u.flat_shard.data), "v": torch.zeros_like(u.flat_shard.data),
                           "step": 0}
        self._shards = nn.ParameterList([u.flat_shard for u in self._units])
        self._prefetch_stream = None
        if prefetch and device.type == "cuda" and self.world_size > 1:
            st = getattr(self, "_gather_state", None)
            self._prefetch_stream = st["stream"] if st is not None else torch.cuda.Stream(device=device)
        self._callback_queued = False
        self._register_hooks()

    def _build_units(self, root, unit_types, reshard_after_forward, reshard_root, device) -> list[_FSDPUnit]:
        units: list[_FSDPUnit] = []
        claimed: set[int] = set()
        for name, m in root.named_modules():
            if m is root or not isinstance(m, unit_types):
                continue
            params = [p for p in m.parameters() if id(p) not in claimed]
            if not params:
                continue
            claimed.update(id(p) for p in params)
            units.append(_FSDPUnit(m, params, self.process_group, self.policy, reshard_after_forward,
                                   device, name or "root", align=self._align))
        rest = [p for p in root.parameters() if id(p) not in claimed]
        if rest:
            # The root unit (embeddings, final norm, head) is needed at both ends
            # of backward, so by default it stays gathered after forward.
            units.append(_FSDPUnit(root, rest, self.process_group, self.policy, reshard_root, device, "<root>",
                                   align=self._align))
        if not units:
            raise ValueError("FSDP wrapped a module with no parameters")
        return units

    def _register_hooks(self) -> None:
        order = [u for u in self._units if u.module is not self.module]
        nxt = {id(u): (order[i + 1] if i + 1 < len(order) else None) for i, u in enumerate(order)}
        prv = {id(u): (order[i - 1] if i > 0 else None) for i, u in enumerate(order)}
        for u in self._units:
            u._hook_handles.append(u.module.register_forward_pre_hook(self._pre_forward(u, nxt.get(id(u)))))
            u._hook_handles.append(u.module.register_forward_hook(self._post_forward(u)))
            if u.reshard_after_forward:
                u._hook_handles.append(
                    u.module.register_full_backward_pre_hook(self._pre_backward(u, prv.get(id(u)))))
            for p in u.params:
                if p.requires_grad:
                    u._hook_handles.append(p.register_post_accumulate_grad_hook(self._grad_ready(u)))
                    u._hook_handles.append(gradsink.add_ready_hook(p, self._grad_ready(u)))

    def _prefetch(self, unit: _FSDPUnit | None) -> None:
        if unit is not None and self._prefetch_stream is not None:
            unit.prefetch(self._prefetch_stream)

    def _pre_forward(self, unit, following):
        def hook(module, args):
            unit.unshard()
            if torch.is_grad_enabled():
                unit.arm_gradient_reduction()
            self._prefetch(following)
        return hook

    def _post_forward(self, unit):
        def hook(module, args, output):
            if unit.reshard_after_forward or not torch.is_grad_enabled():
                unit.reshard()
        return hook

    def _pre_backward(self, unit, preceding):
        def hook(module, grad_output):
            unit.unshard()
            self._prefetch(preceding)
        return hook

    def _grad_ready(self, unit):
        def hook(param):
            if not self._callback_queued and getattr(self, "_gather_state", None) is not None:
                self._callback_queued = True
                try:
                    torch.autograd.Variable._execution_engine.queue_callback(self._end_of_backward)
                except Exception:  # pragma: no cover - only legal inside backward
                    self._callback_queued = False
            unit.on_param_grad_ready(param, sync=self.require_backward_grad_sync)
        return hook

    def _end_of_backward(self) -> None:
        """The compute stream waits for the reduce-scatters still running on the communication stream."""
        self._callback_queued = False
        self._wait_comm()

    def _wait_comm(self) -> None:
        st = getattr(self, "_gather_state", None)
        if st is not None and st["pending"]:
            torch.cuda.current_stream().wait_stream(st["stream"])
            st["pending"] = False

    # -- public API ----------------------------------------------------------------

    def forward(self, *args, **kwargs):
        return self.module(*args, **kwargs)

    def named_parameters(self, prefix: str = "", recurse: bool = True, remove_duplicate: bool = True):
        """Only the flat shards (``_flat_shard_{i}``): the optimizer must never see the gathered views."""
        for i, u in enumerate(self._units):
            yield f"{prefix}{'.' if prefix else ''}_flat_shard_{i}", u.flat_shard

    def parameters(self, recurse: bool = True):
        for _, p in self.named_parameters(recurse=recurse):
            yield p

    @contextmanager
    def no_sync(self) -> Iterator[None]:
        """Accumulate full gradients locally (memory-hungry: every unit keeps its full grads)."""
        prev = self.require_backward_grad_sync
        self.require_backward_grad_sync = False
        try:
            yield
        finally:
            self.require_backward_grad_sync = prev

    @contextmanager
    def summon_full_params(self) -> Iterator[None]:
        """Gather every unit for the block, restoring each unit's prior state afterwards."""
        was = [u.is_unsharded for u in self._units]
        for u in self._units:
            u.unshard()
        try:
            yield
        finally:
            for u, w in zip(self._units, was, strict=True):
                if not w:
                    u.reshard()

    def finish_gradient_sync(self) -> None:
        """Reduce-scatter units whose gradients were accumulated under ``no_sync``, and order the
        current stream after every reduce-scatter in flight."""
        if self.world_size == 1:
            return
        for u in self._units:
            if any(p.grad is not None or getattr(p, "_md_grad_written", False) for p in u.params):
                u.reduce_scatter_grads()
                if u.reshard_after_forward:
                    u.reshard()
        self._wait_comm()

    def memory_summary(self) -> dict[str, float]:
        total = sum(u.total_numel for u in self._units)
        sharded = sum(u.shard_numel for u in self._units)
        sb = self._units[0].flat_shard.element_size()
        largest = max(u.total_numel for u in self._units)
        pb = self.policy.param_dtype.itemsize
        mb = 1024**2
        return {
            "params_total_M": total / 1e6,
            "shard_params_MB": sharded * sb / mb,
            "replicated_params_MB": total * sb / mb,
            "fsdp_state_MB": sharded * sb * 4 / mb,  # params + grads + Adam m, v
            "ddp_state_MB": total * sb * 4 / mb,
            "transient_gather_MB": largest * pb / mb,
            "num_units": len(self._units),
        }

    def unit_summary(self) -> list[tuple[str, int, int]]:
        return [(u.name, u.total_numel, u.shard_numel) for u in self._units]

    def __getattr__(self, name: str):
        try:
            return super().__getattr__(name)
        except AttributeError:
            return getattr(self.module, name)


FSDP = FullyShardedDataParallel
