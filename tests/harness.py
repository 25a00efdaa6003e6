"""Multi-process test harness: N spawned processes on Gloo/CPU plus single-process oracles.

Every distributed claim is checked by running the distributed code in ``world``
processes and comparing with a single-process reference built from the same
seeds (the reference's strategy, tests/common.py).  Gloo exercises the same
``torch.distributed`` path as NCCL — group construction, collective order,
autograd hooks — but not NCCL's kernels or stream ordering; the GPU tier
covers those.
"""

from __future__ import annotations

import os
import tempfile
from collections.abc import Callable

import torch
import torch.distributed as dist
import torch.multiprocessing as mp


def _worker(rank: int, world: int, store: str, fn: Callable, args: tuple) -> None:
    os.environ.update(RANK=str(rank), WORLD_SIZE=str(world), LOCAL_RANK=str(rank))
    torch.set_num_threads(1)
    dist.init_process_group("gloo", init_method=f"file://{store}", rank=rank, world_size=world)
    torch.manual_seed(0)
    try:
        fn(rank, world, *args)
    finally:
        dist.barrier()
        dist.destroy_process_group()


def run_distributed(fn: Callable, world: int = 2, *args) -> None:
    """Run module-level ``fn(rank, world, *args)`` in ``world`` spawned Gloo processes."""
    with tempfile.TemporaryDirectory() as tmp:
        mp.spawn(_worker, args=(world, os.path.join(tmp, "store"), fn, args), nprocs=world, join=True)


def solo_group(rank: int, world: int):
    """A size-1 group holding only this rank (``new_group`` is collective, so all ranks loop)."""
    mine = None
    for r in range(world):
        g = dist.new_group([r])
        if r == rank:
            mine = g
    return mine


def assert_close(actual, expected, msg: str, tol: float = 1e-5) -> None:
    """Max-abs difference relative to ``max(|expected|, 1)`` must stay below ``tol``."""
    a, e = actual.detach().float(), expected.detach().float()
    if a.shape != e.shape:
        raise AssertionError(f"{msg}: shape {tuple(a.shape)} != {tuple(e.shape)}")
    err = (a - e).abs().max().item() if a.numel() else 0.0
    rel = err / max(e.abs().max().item() if e.numel() else 0.0, 1.0)
    if rel > tol:
        raise AssertionError(f"{msg}: max abs diff {err:.3e}, relative {rel:.3e} > {tol:.1e}")


def all_ranks_agree(t: torch.Tensor, group=None) -> bool:
    parts = [torch.empty_like(t) for _ in range(dist.get_world_size(group))]
    dist.all_gather(parts, t.contiguous(), group=group)
    return all(torch.equal(parts[0], p) for p in parts[1:])
