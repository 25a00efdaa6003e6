"""Optimizers.

:class:`FusedAdamW` is ``torch.optim.AdamW`` (same hyper-parameters, same
update, same ``state_dict`` keys ``step``/``exp_avg``/``exp_avg_sq``) executed
as one multi-tensor sm_100a kernel per parameter group (csrc/optim.cu).  The
kernel also refreshes the bf16 shadow weights the fused GEMMs read, so the
next forward does not pay for a separate cast.  Off CUDA it runs the same
arithmetic with torch ops, so CPU tests exercise identical semantics.
"""

from __future__ import annotations

import math

import torch

from .ops import _native as nat
from .ops import grads as gradsink

__all__ = ["FusedAdamW"]


class FusedAdamW(torch.optim.Optimizer):
    def __init__(self, params, lr: float = 1e-3, betas=(0.9, 0.999), eps: float = 1e-8,
                 weight_decay: float = 1e-2):
        if lr < 0 or eps < 0 or not (0 <= betas[0] < 1 and 0 <= betas[1] < 1):
            raise ValueError("invalid AdamW hyper-parameters")
        super().__init__(params, dict(lr=lr, betas=betas, eps=eps, weight_decay=weight_decay))
        self._tables: dict[int, tuple] = {}

    # -- state ----------------------------------------------------------------------

    def _state(self, p: torch.Tensor) -> dict:
        st = self.state[p]
        if not st:
            st["step"] = torch.zeros((), dtype=torch.float32)
            st["exp_avg"] = torch.zeros_like(p, memory_format=torch.contiguous_format)
            st["exp_avg_sq"] = torch.zeros_like(p, memory_format=torch.contiguous_format)
        return st

    # -- step -----------------------------------------------------------------------

    @torch.no_grad()
    def step(self, closure=None):
        loss = None
        if closure is not None:
            with torch.enable_grad():
                loss = closure()
        for gi, group in enumerate(self.param_groups):
            params = [p for p in group["params"] if p.grad is not None]
            if not params:
                continue
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
            if fused:
                # Parameters whose gradient all-reduce is still in flight (DDP with
                # defer_last_buckets) are updated last, after waiting on its event.
                late = [p for p in fused if getattr(p, "_md_grad_event", None) is not None]
                if late:
                    early = [p for p in fused if getattr(p, "_md_grad_event", None) is None]
                    if early:
                        self._fused_update((gi, 0), early, lr, b1, b2, eps, wd, bc1, bc2_sqrt)
                    for ev in {id(p._md_grad_event): p._md_grad_event for p in late}.values():
                        torch.cuda.current_stream().wait_event(ev)
                    for p in late:
                        p._md_grad_event = None
                    self._fused_update((gi, 1), late, lr, b1, b2, eps, wd, bc1, bc2_sqrt)
                else:
                    self._fused_update(gi, fused, lr, b1, b2, eps, wd, bc1, bc2_sqrt)
                self._ensure_grad_buffers()
            for p in rest:
                st = self.state[p]
                g = p.grad.to(p.dtype)
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

    def _fused_update(self, gi, params, lr, b1, b2, eps, wd, bc1, bc2_sqrt) -> None:
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
            table = torch.tensor(rows, dtype=torch.int64).to(dev)
            chunks = [(i, c) for i, p in enumerate(params) for c in range(-(-p.numel() // chunk))]
            chunk_t = torch.tensor(chunks, dtype=torch.int32).to(dev)
            cached = (key, table, chunk_t, len(chunks))
            self._tables[gi] = cached
        _, table, chunk_t, n = cached
        rc = lib.md_adamw(table.data_ptr(), chunk_t.data_ptr(), n, lr, b1, b2, eps, wd, bc1, bc2_sqrt,
                          None, None, 0, nat.stream_ptr())
        nat.check(rc, "md_adamw")
        for p in params:
            if getattr(p, _SHADOW, None) is not None:
                setattr(p, _SHADOW_VER, p._version)
