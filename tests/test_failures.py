"""Failure detection on the host (Gloo/CPU ranks; no GPU is faulted, trapped or hung).

* a parameter-layout mismatch between ranks is caught at DDP / FSDP construction,
  on every rank, before any collective that depends on the layout;
* a rank that never joins a collective makes the others fail at the process-group
  timeout instead of waiting forever;
* a rank that raises propagates its exception to the launcher.

The device-side counterpart (bounded waits in the fused kernels returning a
status the host turns into ``CommTimeoutError``) is tests/test_timeouts_gpu.py.
"""

from __future__ import annotations

import time
from datetime import timedelta

import pytest
import torch
import torch.distributed as dist
from torch import nn

import minidist as md

from .harness import run_distributed


def _layout_mismatch(rank, world, which):
    hidden = 16 if rank == 0 else 24  # rank 1 builds a different model
    model = nn.Sequential(nn.Linear(8, hidden), nn.Linear(hidden, 4))
    with pytest.raises(RuntimeError, match="parameter layout differs"):
        if which == "ddp":
            md.DistributedDataParallel(model)
        else:
            md.FullyShardedDataParallel(model, device=torch.device("cpu"))


@pytest.mark.parametrize("which", ["ddp", "fsdp"])
def test_layout_mismatch_is_caught_on_every_rank(which):
    run_distributed(_layout_mismatch, 2, which)


def _missing_rank(rank, world):
    g = dist.new_group(list(range(world)), timeout=timedelta(seconds=3))
    if rank == 0:
        t = torch.ones(4)
        t0 = time.monotonic()
        with pytest.raises(RuntimeError):
            dist.all_reduce(t, group=g)  # rank 1 never joins
        assert time.monotonic() - t0 < 60
    else:
        time.sleep(6)  # longer than the group timeout, then carry on to the harness barrier


def test_rank_that_never_joins_times_out():
    run_distributed(_missing_rank, 2)


def _raising_rank(rank, world):
    if rank == 1:
        raise ValueError("injected failure on rank 1")


def test_rank_exception_propagates():
    with pytest.raises(Exception, match="injected failure on rank 1"):
        run_distributed(_raising_rank, 2)
