"""Whole training steps as CUDA graphs.

A GPT-2-small step on one B200 is ~320 kernel launches; launched one by one
from Python, the gaps between them cost ~5% of the step.  :class:`GraphedStep`
captures ``fn(*inputs)`` -- forward, backward, gradient collectives and the
optimizer -- once as a CUDA graph and replays it: one launch per step, the
inputs copied into fixed device buffers first.

What makes a step replayable here:

* the sm_100a kernels take their pointers and shapes as launch parameters and
  run on the current stream (the capture stream during capture); activations
  come from the graph's private memory pool, so every replay sees the same
  addresses;
* the peer-memory collectives (DDP bucket all-reduce, FSDP reduce-scatter /
  all-gather, fused GEMM + all-reduce) count their barrier epochs on the
  device, so a replay waits for the peers' replay rather than for flags left by
  the previous step;
* :class:`~minidist.optim.FusedAdamW` must be built with ``capturable=True``:
  its step count and learning rate live in device memory;
* NCCL calls (pipeline send / recv, fallback collectives) are captured as graph
  nodes by NCCL itself.

Requirements on ``fn``: no host synchronisation (``.item()``, ``.cpu()``), no
data-dependent Python control flow, and ``torch.autocast(..., cache_enabled=False)``
if it uses autocast.  The reference has no counterpart (it runs eagerly,
examples/train_gpt.py); this is the B200 path's launch-overhead answer in place
of a tracing compiler.
"""

from __future__ import annotations

from collections.abc import Callable, Sequence

import torch

__all__ = ["GraphedStep"]


class GraphedStep:
    """``fn(*inputs)`` captured as one CUDA graph.

    ``example_inputs`` fix the input shapes and dtypes (they are copied into the
    graph's static input buffers).  Construction runs ``warmup`` eager steps on a
    side stream (lazy initialisation, optimizer state, gradient buffers) and then
    captures one step; the captured step does not execute, so the model advances
    by ``warmup`` steps here.  ``step(*inputs)`` copies ``inputs`` into the static
    buffers (device-to-device, or host-to-device from pinned memory without a
    host sync), refreshes the ``optimizers``' device hyper-parameters and replays
    the graph.  It returns ``fn``'s output tensors, which the next replay
    overwrites.
    """

    def __init__(self, fn: Callable, example_inputs: Sequence[torch.Tensor], warmup: int = 2,
                 optimizers: Sequence = (), pool=None):
        if not torch.cuda.is_available():
            raise RuntimeError("GraphedStep needs CUDA")
        if warmup < 1:
            raise ValueError("at least one eager warm-up step is needed before capture")
        for opt in optimizers:
            if hasattr(opt, "capturable") and not opt.capturable:
                raise ValueError(f"{type(opt).__name__} must be built with capturable=True")
        self.fn = fn
        self.optimizers = list(optimizers)
        self.static_inputs = [t.detach().to("cuda").clone() for t in example_inputs]
        side = torch.cuda.Stream()
        side.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(side):
            for _ in range(warmup):
                fn(*self.static_inputs)
        torch.cuda.current_stream().wait_stream(side)
        torch.cuda.synchronize()
        for opt in self.optimizers:
            if hasattr(opt, "sync_hyperparams"):
                opt.sync_hyperparams()
        self.graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self.graph, pool=pool):
            self.static_outputs = fn(*self.static_inputs)
        torch.cuda.synchronize()
        self.replays = 0

    def __call__(self, *inputs: torch.Tensor):
        if len(inputs) != len(self.static_inputs):
            raise ValueError(f"expected {len(self.static_inputs)} inputs, got {len(inputs)}")
        for dst, src in zip(self.static_inputs, inputs, strict=True):
            if src.data_ptr() != dst.data_ptr():
                dst.copy_(src, non_blocking=True)
        for opt in self.optimizers:
            if hasattr(opt, "sync_hyperparams"):
                opt.sync_hyperparams()
        self.graph.replay()
        self.replays += 1
        return self.static_outputs

    step = __call__

    def release(self) -> None:
        """Free the graph (before ``destroy_process_group`` when it holds NCCL calls)."""
        self.graph.reset()
        self.static_outputs = None
