"""Optimizers.

:class:`FusedAdamW` is ``torch.optim.AdamW`` (same hyper-parameters, same
update, same ``state_dict`` keys ``step``/``exp_avg``/``exp_avg_sq``) executed
as one multi-tensor sm_100a kernel per parameter group (csrc/optim.cu).  The
kernel also refreshes the bf16 shadow weights the fused GEMMs read, so the
next forward does not pay for a separate cast.  Off CUDA it runs the same
arithmetic with torch ops, so CPU tests exercise identical semantics.

``capturable=True`` keeps each group's learning rate and step count in device
memory ([lr, t]; the kernel computes the bias corrections), so a training step
captured in a CUDA graph (:class:`minidist.graphs.GraphedStep`) advances the
step on every replay; :meth:`FusedAdamW.sync_hyperparams` refreshes the device
learning rate from ``param_groups`` between replays.
"""

from __future__ import annotations

import math

import torch

from .ddp import wait_handle
from .ops import _native as nat
from .ops import grads as gradsink

__all__ = ["FusedAdamW"]


class FusedAdamW(torch.optim.Optimizer):
    # Parameters whose DDP all-reduce is still in flight (``_md_grad_event``) are
    # updated last, after waiting on exactly their handle (DistributedDataParallel's
    # ``defer_last_buckets``); the global step guard in minidist.ddp leaves them to us.
    honours_grad_events = True

    def __init__(self, params, lr: float = 1e-3, betas=(0.9, 0.999), eps: float = 1e-8,
                 weight_decay: float = 1e-2, capturable: bool = False):
        if lr < 0 or eps < 0 or not (0 <= betas[0] < 1 and 0 <= betas[1] < 1):
            raise ValueError("invalid AdamW hyper-parameters")
        super().__init__(params, dict(lr=lr, betas=betas, eps=eps, weight_decay=weight_decay))
        self._tables: dict[int, tuple] = {}
        self.capturable = capturable
        self._hp: dict[int, torch.Tensor] = {}  # capturable: device [lr, step] per group
        self._hp_lr: dict[int, float] = {}

    def sync_hyperparams(self) -> None:
        """Copy each group's current ``lr`` into its device slot (capturable mode; call between
        graph replays -- it launches work, so not while a graph is being captured)."""
        for gi, hp in self._hp.items():
            lr = float(self.param_groups[gi]["lr"])
            if self._hp_lr.get(gi) != lr:
                hp[0:1].fill_(lr)
                self._hp_lr[gi] = lr

    def state_dict(self):
        # In capturable mode the step count advances on the device; bring it to the host state.
        for gi, hp in self._hp.items():
            t = float(hp[1].item())
            for p in self.param_groups[gi]["params"]:
                st = self.state.get(p)
                if st and "step" in st:
                    st["step"].fill_(t)
        return super().state_dict()

    # -- state ----------------------------------------------------------------------

    def _state(self, p: torch.Tensor) -> dict:
        st = self.state[p]
        if not st:
            st["step"] = torch.zeros((), dtype=torch.float32)
            st["exp_avg"] = torch.zeros_like(p, memory_format=torch.contiguous_format)
            st["exp_avg_sq"] = torch.zeros_like(p, memory_format=torch.contiguous_format)
        return st

    def _init_states(self, params) -> None:
        """First step of CUDA fp32 parameters: their moments as views of two flat zeroed buffers
        (two fills for the whole group instead of two per parameter; 16-byte-aligned slices)."""
        todo = [p for p in params if not self.state[p] and p.is_cuda and p.dtype == torch.float32]
        if not todo:
            return
        sizes = [(p.numel() + 3) // 4 * 4 for p in todo]
        flat = torch.zeros(2, sum(sizes), dtype=torch.float32, device=todo[0].device)
        off = 0
        for p, n in zip(todo, sizes):
            st = self.state[p]
            st["step"] = torch.zeros((), dtype=torch.float32)
            st["exp_avg"] = flat[0, off: off + p.numel()].view_as(p)
            st["exp_avg_sq"] = flat[1, off: off + p.numel()].view_as(p)
            off += n

    # -- step -----------------------------------------------------------------------

    @torch.no_grad()
    def check_nonfinite(self, flag: torch.Tensor) -> None:
        """Set device ``flag`` (float32 ``[1]``) to 1 if any gradient is inf / NaN, without a host
        synchronisation (one read-only multi-tensor pass per parameter group; CPU parameters are
        checked with torch ops)."""
        for gi, group in enumerate(self.param_groups):
            params = [p for p in group["params"] if p.grad is not None]
            fused = [p for p in params if p.is_cuda and p.dtype == torch.float32 and p.grad.dtype == torch.float32]
            fused_ids = {id(p) for p in fused}
            for p in params:
                if id(p) not in fused_ids:
                    flag.add_((~torch.isfinite(p.grad)).any().to(flag.dtype).to(flag.device))
            self._init_states(fused)  # the kernel table points at the moments too
            if fused:
                for key, part in self._partitions(gi, fused):
                    table, chunk_t, n = self._table(key, part)
                    nat.check(nat.lib().md_nonfinite(table.data_ptr(), chunk_t.data_ptr(), n, flag.data_ptr(),
                                                     nat.stream_ptr()), "md_nonfinite")

    def _partitions(self, gi, fused):
        late = [p for p in fused if getattr(p, "_md_grad_event", None) is not None]
        if not late:
            return [(gi, fused)]
        early = [p for p in fused if getattr(p, "_md_grad_event", None) is None]
        return [((gi, 0), early), ((gi, 1), late)] if early else [((gi, 1), late)]

    @torch.no_grad()
    def step(self, closure=None, *, inv_scale: torch.Tensor | None = None, skip: torch.Tensor | None = None):
        """One AdamW step.  ``inv_scale`` / ``skip`` (device float32 ``[1]``, from
        :class:`minidist.amp.DistributedGradScaler`): gradients are multiplied by ``inv_scale``
        inside the update kernel, and the whole update is skipped on the device when ``skip``
        is nonzero -- the loss scaler's unscale and overflow skip with no extra pass over the
        gradients and no host synchronisation."""
        loss = None
        if closure is not None:
            with torch.enable_grad():
                loss = closure()
        self._scaler_ptrs = (None if inv_scale is None else inv_scale.data_ptr(),
                             None if skip is None else skip.data_ptr())
        for gi, group in enumerate(self.param_groups):
            params = [p for p in group["params"] if p.grad is not None]
            if not params:
                continue
            self._init_states(params)
            states = [self._state(p) for p in params]
            # One multi-tensor op for every parameter's step count (a per-tensor
            # loop of CPU adds cost ~0.6 ms of host time per step at GPT-2 size).
            torch._foreach_add_([st["step"] for st in states], 1.0)
            t = float(states[0]["step"])
            b1, b2 = group["betas"]
            lr, eps, wd = group["lr"], group["eps"], group["weight_decay"]
            bc1 = 1.0 - b1**t
            bc2_sqrt = math.sqrt(1.0 - b2**t)
            cuda = [p.is_cuda and p.dtype == torch.float32 and p.grad.dtype == torch.float32 for p in params]
            fused = [p for p, c in zip(params, cuda) if c]
            rest = [p for p, c in zip(params, cuda) if not c]
            hp = None
            if self.capturable and fused:
                hp = self._hp.get(gi)
                if hp is None:
                    if torch.cuda.is_current_stream_capturing():
                        raise RuntimeError("FusedAdamW(capturable=True) needs one eager step before capture")
                    hp = torch.tensor([lr, t - 1.0], dtype=torch.float32, device=fused[0].device)
                    self._hp[gi], self._hp_lr[gi] = hp, float(lr)
                if not torch.cuda.is_current_stream_capturing():
                    self.sync_hyperparams()
                hp[1:2].add_(1.0)
            if rest and torch.cuda.is_available() and torch.cuda.is_current_stream_capturing():
                raise RuntimeError("FusedAdamW: only CUDA fp32 parameters can be stepped inside a CUDA graph")
            if fused:
                # Parameters whose gradient all-reduce is still in flight (DDP with
                # defer_last_buckets) are updated last, after waiting on its event.
                late = [p for p in fused if getattr(p, "_md_grad_event", None) is not None]
                if late:
                    early = [p for p in fused if getattr(p, "_md_grad_event", None) is None]
                    if early:
                        self._fused_update((gi, 0), early, lr, b1, b2, eps, wd, bc1, bc2_sqrt, hp)
                    for ev in {id(p._md_grad_event): p._md_grad_event for p in late}.values():
                        wait_handle(ev)
                    for p in late:
                        p._md_grad_event = None
                    self._fused_update((gi, 1), late, lr, b1, b2, eps, wd, bc1, bc2_sqrt, hp)
                else:
                    self._fused_update(gi, fused, lr, b1, b2, eps, wd, bc1, bc2_sqrt, hp)
                self._ensure_grad_buffers()
            for ev in {id(h): h for h in (getattr(p, "_md_grad_event", None) for p in rest) if h is not None}.values():
                wait_handle(ev)
            if rest and skip is not None and bool(skip.item()):
                rest = []
            for p in rest:
                p._md_grad_event = None
                st = self.state[p]
                g = p.grad.to(p.dtype)
                if inv_scale is not None:
                    g = g * inv_scale.to(g.device)
                p.mul_(1 - lr * wd)
                st["exp_avg"].mul_(b1).add_(g, alpha=1 - b1)
                st["exp_avg_sq"].mul_(b2).addcmul_(g, g, value=1 - b2)
                denom = st["exp_avg_sq"].sqrt().div_(bc2_sqrt).add_(eps)
                p.addcdiv_(st["exp_avg"], denom, value=-lr / bc1)
        return loss

    def _ensure_grad_buffers(self) -> None:
        """Give every CUDA fp32 parameter without one a persistent gradient buffer.

        Fused kernels write gradients into these views (ops/grads.py), so the
        gradient pointers stay fixed from step to step and the device-side
        parameter table is built once.  Parameters that a wrapper (DDP) has
        already given a buffer keep it.
        """
        if getattr(self, "_grad_buffers_done", False):
            return
        self._grad_buffers_done = True
        todo = [p for g in self.param_groups for p in g["params"]
                if p.is_cuda and p.dtype == torch.float32 and gradsink.main_grad(p) is None]
        if not todo:
            return
        align = 64
        sizes = [(p.numel() + align - 1) // align * align for p in todo]
        flat = torch.zeros(sum(sizes), dtype=torch.float32, device=todo[0].device)
        off = 0
        for p, n in zip(todo, sizes):
            view = flat[off: off + p.numel()].view_as(p)
            if p.grad is not None:
                view.copy_(p.grad)
                p.grad = view
            gradsink.set_main_grad(p, view)
            off += n
        self._grad_flat = flat

    def _fused_update(self, gi, params, lr, b1, b2, eps, wd, bc1, bc2_sqrt, hp=None) -> None:
        from .models.fused_gpt import _SHADOW

        table, chunk_t, n = self._table(gi, params)
        inv_ptr, skip_ptr = getattr(self, "_scaler_ptrs", (None, None))
        rc = nat.lib().md_adamw(table.data_ptr(), chunk_t.data_ptr(), n, lr, b1, b2, eps, wd, bc1, bc2_sqrt,
                                inv_ptr, skip_ptr, 0, nat.stream_ptr(), None if hp is None else hp.data_ptr())
        nat.check(rc, "md_adamw")
        for p in params:
            if getattr(p, _SHADOW, None) is not None:
                setattr(p, "_md_bf16_ver", p._version)

    def _table(self, gi, params):
        """Device (tensor, chunk) table of ``params`` for the multi-tensor kernels, cached per key
        while the pointers stay the same."""
        from .models.fused_gpt import _SHADOW, _SHADOW_VER

        lib = nat.lib()
        rows, key = [], []
        for p in params:
            st = self.state[p]
            g = p.grad if p.grad.is_contiguous() else p.grad.contiguous()
            sh = getattr(p, _SHADOW, None)
            if sh is not None and (sh.shape != p.shape or getattr(p, _SHADOW_VER, None) != p._version):
                sh = None  # stale shadow: let the next forward recast it
            ptrs = (p.data_ptr(), g.data_ptr(), st["exp_avg"].data_ptr(), st["exp_avg_sq"].data_ptr(),
                    sh.data_ptr() if sh is not None else 0, p.numel())
            rows.append(ptrs)
            key.append(ptrs)
        key = tuple(key)
        cached = self._tables.get(gi)
        dev = params[0].device
        if cached is None or cached[0] != key:
            chunk = lib.md_adamw_chunk()
            chunks = [(i, c) for i, p in enumerate(params) for c in range(-(-p.numel() // chunk))]
            # Pinned sources: a copy from pageable memory is not allowed inside a graph capture.
            table_h = torch.tensor(rows, dtype=torch.int64).pin_memory()
            chunk_h = torch.tensor(chunks, dtype=torch.int32).pin_memory()
            table = table_h.to(dev, non_blocking=True)
            chunk_t = chunk_h.to(dev, non_blocking=True)
            cached = (key, table, chunk_t, len(chunks), table_h, chunk_h)
            self._tables[gi] = cached
        return cached[1], cached[2], cached[3]
