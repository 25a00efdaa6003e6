"""Where fused kernels put parameter gradients, and how wrappers hear about them.

The fused CUDA ops write weight gradients straight from the GEMM epilogue
(fp32, accumulating when a gradient already exists) instead of returning them
through autograd, which would cost an extra full-size write plus an
accumulate.  Autograd's ``post_accumulate_grad_hook`` therefore does not fire
for those parameters, so this module provides the equivalent protocol:

* :func:`grad_destination` — the tensor a kernel should write ``p``'s gradient
  into and whether to accumulate.  It prefers ``p.grad``; otherwise the
  "main grad" view a wrapper registered (a DDP bucket slice, see ddp.py), so
  gradients land in the communication buffer with no copy.
* :func:`mark_ready` — called once the kernel producing ``p``'s gradient has
  been enqueued; runs the hooks wrappers registered with :func:`add_ready_hook`
  (DDP bucket accounting, FSDP reduce-scatter triggering).

Parameters whose gradients do flow through autograd keep using torch's hooks;
DDP and FSDP register both kinds and each parameter fires exactly one.
"""

from __future__ import annotations

from collections.abc import Callable

import torch

_MAIN = "_md_main_grad"
_HOOKS = "_md_ready_hooks"


def set_main_grad(p: torch.Tensor, view: torch.Tensor | None) -> None:
    setattr(p, _MAIN, view)


def main_grad(p: torch.Tensor) -> torch.Tensor | None:
    return getattr(p, _MAIN, None)


class _Handle:
    def __init__(self, p: torch.Tensor, fn: Callable):
        self._p, self._fn = p, fn

    def remove(self) -> None:
        hooks = getattr(self._p, _HOOKS, None)
        if hooks and self._fn in hooks:
            hooks.remove(self._fn)


def add_ready_hook(p: torch.Tensor, fn: Callable[[torch.Tensor], None]) -> _Handle:
    hooks = getattr(p, _HOOKS, None)
    if hooks is None:
        hooks = []
        setattr(p, _HOOKS, hooks)
    hooks.append(fn)
    return _Handle(p, fn)


def grad_destination(p: torch.Tensor, dtype: torch.dtype = torch.float32) -> tuple[torch.Tensor, bool]:
    """``(dst, accumulate)`` for writing ``p``'s gradient; sets ``p.grad`` to ``dst``."""
    g = p.grad
    if g is not None:
        return g, True
    mg = main_grad(p)
    if mg is not None and mg.dtype == dtype:
        p.grad = mg
        return mg, False
    g = torch.empty(p.shape, dtype=dtype, device=p.device)
    p.grad = g
    return g, False


def mark_ready(p: torch.Tensor) -> None:
    for fn in list(getattr(p, _HOOKS, ()) or ()):
        fn(p)
