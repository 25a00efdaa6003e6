"""Loss-scaler decisions are unanimous across ranks (host-side fault injection with inf/NaN)."""

from __future__ import annotations

import pytest
import torch
import torch.distributed as dist

from minidist.amp import DistributedGradScaler, resolve_precision

from .harness import run_distributed


def _model():
    torch.manual_seed(0)
    m = torch.nn.Linear(4, 4)
    return m, torch.optim.SGD(m.parameters(), lr=0.1)


def _overflow_on_rank0(rank, world):
    m, opt = _model()
    sc = DistributedGradScaler(init_scale=1024.0)
    for p in m.parameters():
        p.grad = torch.ones_like(p)
    if rank == 0:
        next(iter(m.parameters())).grad[0, 0] = float("inf")
    before = [p.detach().clone() for p in m.parameters()]
    stepped = sc.step(opt)
    sc.update()
    assert not stepped, f"[rank {rank}] stepped despite rank 0's overflow"
    assert all(torch.equal(p.detach(), b) for p, b in zip(m.parameters(), before))
    assert sc.scale == 512.0 and sc.num_skipped == 1


def _growth(rank, world):
    m, opt = _model()
    sc = DistributedGradScaler(init_scale=1024.0, growth_interval=2)
    for _ in range(2):
        for p in m.parameters():
            p.grad = torch.full_like(p, 2.0) * sc.scale
        assert sc.step(opt)
        sc.update()
    assert sc.scale == 2048.0 and sc.num_skipped == 0


def _unscale(rank, world):
    m, opt = _model()
    sc = DistributedGradScaler(init_scale=256.0)
    for p in m.parameters():
        p.grad = torch.full_like(p, 3.0) * sc.scale
    assert not sc.unscale_(opt)
    sc.unscale_(opt)  # second call must not divide again
    for p in m.parameters():
        assert torch.allclose(p.grad, torch.full_like(p.grad, 3.0))


def _history(rank, world):
    m, opt = _model()
    sc = DistributedGradScaler(init_scale=4096.0, growth_interval=2)
    for bad in [0, 2, 2, 1, 1]:  # rank that sees a NaN each step (2 = none)
        for p in m.parameters():
            p.grad = torch.ones_like(p)
        if rank == bad:
            next(iter(m.parameters())).grad[0, 0] = float("nan")
        sc.step(opt)
        sc.update()
    s = torch.tensor([sc.scale])
    parts = [torch.empty_like(s) for _ in range(world)]
    dist.all_gather(parts, s)
    assert all(torch.equal(parts[0], x) for x in parts)


def test_overflow_on_one_rank_skips_everywhere():
    run_distributed(_overflow_on_rank0, 2)


def test_clean_steps_grow_the_scale():
    run_distributed(_growth, 2)


def test_unscale_is_idempotent():
    run_distributed(_unscale, 2)


def test_scale_stays_in_sync_across_ranks():
    run_distributed(_history, 3)


def test_resolve_precision():
    cpu = torch.device("cpu")
    assert not resolve_precision("fp32", cpu).enabled
    bf16 = resolve_precision("bf16", cpu)
    assert bf16.dtype == torch.bfloat16 and not bf16.needs_grad_scaler
    assert resolve_precision("auto", cpu).dtype == torch.bfloat16
    with pytest.raises(ValueError):
        resolve_precision("fp16", cpu)
    with pytest.raises(ValueError):
        resolve_precision("int4", cpu)


def test_disabled_scaler_is_transparent():
    m, opt = _model()
    sc = DistributedGradScaler(enabled=False)
    loss = torch.tensor(2.0)
    assert sc.scale_loss(loss) is loss and sc.scale == 1.0
    for p in m.parameters():
        p.grad = torch.ones_like(p)
    assert sc.step(opt)
