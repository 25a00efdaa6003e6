"""Mixed precision: the precision policy and a loss scaler whose decisions are collective.

bf16 keeps fp32's 8-bit exponent, so bf16 training needs no loss scaling and
is the product path on B200 (every hand-written kernel takes bf16 operands and
accumulates in fp32).  fp16 has the mantissa but not the range, so it needs a
dynamic loss scale.

The scaler's overflow test is local to a rank, yet under FSDP and tensor
parallelism each rank holds a *different* piece of the gradient: an inf in one
shard is invisible to the others.  If only that rank skipped the step the
replicas would diverge silently.  :class:`DistributedGradScaler` therefore
all-reduces the ``found_inf`` flag with MAX over the group before anyone acts on
it, and every rank then runs identical scale arithmetic (reference
amp.py:26-49, 195-223).
"""

from __future__ import annotations

from contextlib import nullcontext
from dataclasses import dataclass

import torch
import torch.distributed as dist

from . import comm

__all__ = ["PrecisionConfig", "DistributedGradScaler", "resolve_precision"]

_NAMES = {"fp32": torch.float32, "bf16": torch.bfloat16, "fp16": torch.float16}


@dataclass
class PrecisionConfig:
    """A run's precision: compute ``dtype``, the autocast device type, and whether it is on."""

    dtype: torch.dtype
    device_type: str
    enabled: bool

    @property
    def needs_grad_scaler(self) -> bool:
        return self.enabled and self.dtype == torch.float16

    def autocast(self):
        """Context for ops that are not routed to the fused kernels (e.g. user modules)."""
        if not self.enabled:
            return nullcontext()
        return torch.autocast(device_type=self.device_type, dtype=self.dtype)

    def __repr__(self) -> str:
        if not self.enabled:
            return "PrecisionConfig(fp32)"
        return f"PrecisionConfig({str(self.dtype).replace('torch.', '')} autocast)"


def resolve_precision(name: str, device: torch.device | None = None) -> PrecisionConfig:
    """``'fp32' | 'fp16' | 'bf16' | 'auto'`` -> :class:`PrecisionConfig`.

    ``auto`` chooses bf16 where the device supports it (every B200 does) and
    fp16 otherwise.  fp16 on CPU is refused: its overflow behaviour would not
    match a GPU run.
    """
    device = device or comm.current_device()
    dev = device.type
    if name == "auto":
        name = "bf16" if (dev != "cuda" or torch.cuda.is_bf16_supported()) else "fp16"
    if name not in _NAMES:
        raise ValueError(f"unknown precision {name!r}")
    if name == "fp16" and dev == "cpu":
        raise ValueError("fp16 autocast is not useful on CPU; use bf16 or fp32")
    dtype = _NAMES[name]
    return PrecisionConfig(dtype, dev, enabled=dtype != torch.float32)


class DistributedGradScaler:
    """Dynamic loss scaling with a group-wide skip decision.

    ``process_group`` must cover every rank that holds part of the gradient —
    for a 3-D run that is the whole world (``None``, the default).  The scale
    halves (``backoff_factor``, floored at ``min_scale``) on an overflow step
    and doubles (``growth_factor``) after ``growth_interval`` clean steps.
    """

    def __init__(
        self,
        init_scale: float = 2.0**16,
        growth_factor: float = 2.0,
        backoff_factor: float = 0.5,
        growth_interval: int = 2000,
        enabled: bool = True,
        process_group: dist.ProcessGroup | None = None,
        min_scale: float = 1.0,
    ):
        self.enabled = enabled
        self.process_group = process_group
        self._scale = float(init_scale)
        self._growth_factor = float(growth_factor)
        self._backoff_factor = float(backoff_factor)
        self._growth_interval = int(growth_interval)
        self._min_scale = float(min_scale)
        self._good_steps = 0
        self._step_found_inf: bool | None = None  # None until unscale_ runs this step
        self.num_skipped = 0
        self.num_steps = 0

    # -- state ----------------------------------------------------------------

    @property
    def scale(self) -> float:
        return self._scale if self.enabled else 1.0

    def state_dict(self) -> dict:
        return {
            "scale": self._scale,
            "good_steps": self._good_steps,
            "num_skipped": self.num_skipped,
            "num_steps": self.num_steps,
        }

    def load_state_dict(self, state: dict) -> None:
        self._scale = float(state["scale"])
        self._good_steps = int(state["good_steps"])
        self.num_skipped = int(state.get("num_skipped", 0))
        self.num_steps = int(state.get("num_steps", 0))

    # -- training-loop surface -------------------------------------------------

    def scale_loss(self, loss: torch.Tensor) -> torch.Tensor:
        return loss * self._scale if self.enabled else loss

    scale_tensor = scale_loss

    @staticmethod
    def _grads(optimizer: torch.optim.Optimizer) -> list[torch.Tensor]:
        return [p.grad for g in optimizer.param_groups for p in g["params"] if p.grad is not None]

    def unscale_(self, optimizer: torch.optim.Optimizer) -> bool:
        """Divide gradients by the scale once per step; return the group-wide overflow flag."""
        if not self.enabled:
            return False
        if self._step_found_inf is not None:
            return self._step_found_inf
        from .ddp import wait_all_deferred

        wait_all_deferred()  # DDP tail buckets still being reduced (defer_last_buckets)
        grads = self._grads(optimizer)
        device = grads[0].device if grads else comm.current_device()
        flag = torch.zeros(1, dtype=torch.float32, device=device)
        inv = 1.0 / self._scale
        if grads and device.type == "cuda":
            # One multi-tensor launch per dtype/device bucket; no host sync per grad.
            inv_t = torch.full((1,), inv, dtype=torch.float32, device=device)
            torch._amp_foreach_non_finite_check_and_unscale_(grads, flag, inv_t)
        else:
            for g in grads:
                g.mul_(inv)
                flag.add_((~torch.isfinite(g)).any().to(flag.dtype))
        if comm.is_distributed() and comm.get_world_size(self.process_group) > 1:
            dist.all_reduce(flag, op=dist.ReduceOp.MAX, group=self.process_group)
        self._step_found_inf = bool(flag.item() > 0)
        return self._step_found_inf

    def step(self, optimizer: torch.optim.Optimizer) -> bool:
        """Apply ``optimizer.step()`` unless the group found an overflow; return whether it stepped.

        With :class:`minidist.optim.FusedAdamW` on CUDA (and ``unscale_`` not called this step)
        the decision stays on the device: a read-only overflow check of the gradients, the
        group-wide MAX of the flag, then the AdamW kernel, which unscales each gradient as it
        reads it and skips the whole update when the flag is set -- no separate unscale pass
        and no host synchronisation here.  The outcome is read in :meth:`update`; this call
        returns ``True`` (the update was issued, conditionally)."""
        self.num_steps += 1
        if not self.enabled:
            optimizer.step()
            return True
        if self._step_found_inf is None and getattr(optimizer, "check_nonfinite", None) is not None:
            grads = self._grads(optimizer)
            if grads and grads[0].is_cuda:
                from .ddp import wait_all_deferred

                wait_all_deferred()  # the check reads every gradient
                flag = torch.zeros(1, dtype=torch.float32, device=grads[0].device)
                optimizer.check_nonfinite(flag)
                if comm.is_distributed() and comm.get_world_size(self.process_group) > 1:
                    dist.all_reduce(flag, op=dist.ReduceOp.MAX, group=self.process_group)
                inv = torch.full((1,), 1.0 / self._scale, dtype=torch.float32, device=flag.device)
                optimizer.step(inv_scale=inv, skip=flag)
                self._device_found_inf = flag
                return True
        if self.unscale_(optimizer):
            self.num_skipped += 1
            return False
        optimizer.step()
        return True

    def update(self) -> None:
        """Adapt the scale from this step's (group-agreed) outcome and reset per-step state."""
        if not self.enabled:
            return
        flag = getattr(self, "_device_found_inf", None)
        if flag is not None:
            self._device_found_inf = None
            self._step_found_inf = bool(flag.item() > 0)
            if self._step_found_inf:
                self.num_skipped += 1
        if self._step_found_inf:
            self._scale = max(self._min_scale, self._scale * self._backoff_factor)
            self._good_steps = 0
        else:
            self._good_steps += 1
            if self._good_steps >= self._growth_interval:
                self._scale *= self._growth_factor
                self._good_steps = 0
        self._step_found_inf = None

    def summary(self) -> str:
        if not self.enabled:
            return "grad scaler disabled (bf16 or fp32)"
        pct = 100.0 * self.num_skipped / max(1, self.num_steps)
        return f"scale={self._scale:g}  skipped={self.num_skipped}/{self.num_steps} ({pct:.1f}%)"
