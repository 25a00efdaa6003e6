"""DDP yields the full-batch gradient whatever the bucketing, overlap or accumulation."""

from __future__ import annotations

import pytest
import torch

from minidist.ddp import DistributedDataParallel
from minidist.models import GPT, GPTConfig

from .harness import assert_close, run_distributed, solo_group

CFG = GPTConfig(vocab_size=64, block_size=16, n_layer=2, n_head=4, n_embd=32)
BATCH = 8


def _data():
    g = torch.Generator().manual_seed(42)
    ids = torch.randint(0, CFG.vocab_size, (BATCH, CFG.block_size), generator=g)
    tgt = torch.randint(0, CFG.vocab_size, (BATCH, CFG.block_size), generator=g)
    return ids, tgt


def _full_batch_grads(solo, ids, tgt):
    m = GPT(CFG, tp_group=solo)
    m(ids, tgt)[1].backward()
    return {n: p.grad.clone() for n, p in m.named_parameters()}


def _check(rank, world, cap, overlap):
    solo = solo_group(rank, world)
    ids, tgt = _data()
    want = _full_batch_grads(solo, ids, tgt)
    model = DistributedDataParallel(GPT(CFG, tp_group=solo), bucket_cap_mb=cap, overlap_with_backward=overlap)
    model(ids.chunk(world)[rank], tgt.chunk(world)[rank])[1].backward()
    for name, p in model.module.named_parameters():
        assert p.grad is not None, name
        assert_close(p.grad, want[name], f"[rank {rank}] cap={cap} overlap={overlap} {name}", tol=2e-5)


def _default(rank, world):
    _check(rank, world, 25.0, True)


def _per_param_buckets(rank, world):
    # A cap below any tensor's size gives one bucket (one collective) per tensor,
    # the configuration most sensitive to launch-order mistakes.
    _check(rank, world, 1e-6, True)


def _single_bucket(rank, world):
    _check(rank, world, 1e6, True)


def _no_overlap(rank, world):
    _check(rank, world, 25.0, False)


def _accumulate(rank, world):
    solo = solo_group(rank, world)
    ids, tgt = _data()
    want = _full_batch_grads(solo, ids, tgt)
    model = DistributedDataParallel(GPT(CFG, tp_group=solo))
    mine = list(zip(ids.chunk(world)[rank].chunk(2), tgt.chunk(world)[rank].chunk(2)))
    with model.no_sync():
        (model(*mine[0])[1] / 2).backward()
    (model(*mine[1])[1] / 2).backward()
    for name, p in model.module.named_parameters():
        assert_close(p.grad, want[name], f"[rank {rank}] accumulated {name}", tol=2e-5)


def _layout(rank, world):
    solo = solo_group(rank, world)
    cap = 0.05
    model = DistributedDataParallel(GPT(CFG, tp_group=solo), bucket_cap_mb=cap)
    summary = model.bucket_summary()
    assert len(summary) > 1
    assert [s[0] for s in summary] == list(range(len(summary)))
    for idx, n, mb in summary:
        assert n >= 1 and (mb <= cap or n == 1), f"bucket {idx}: {mb:.3f} MB over cap"
    params = [p for p in model.module.parameters() if p.requires_grad]
    assert model._buckets[0].params[0] is params[-1], "bucket 0 must start at the last parameter"


def _deferred_with_torch_adamw(rank, world):
    """Deferred tail buckets are invisible to an optimizer that does not ask for them:
    torch AdamW over DDP(defer_last_buckets=2) takes exactly the steps it takes over a DDP
    that waits for every bucket in backward."""
    from minidist import ddp as ddp_mod

    solo = solo_group(rank, world)
    ids, tgt = _data()
    runs = []
    for defer in (0, 2):
        model = DistributedDataParallel(GPT(CFG, tp_group=solo), bucket_cap_mb=0.01, defer_last_buckets=defer)
        opt = torch.optim.AdamW(model.parameters(), lr=1e-2)
        for it in range(3):
            x, y = ids.roll(it, 0).chunk(world)[rank], tgt.roll(it, 0).chunk(world)[rank]
            opt.zero_grad()
            model(x, y)[1].backward()
            if defer:
                assert model._deferred, "the tail buckets should still be in flight after backward"
            opt.step()  # the global step pre-hook waits for them
            assert not model._deferred and model not in ddp_mod._PENDING
        runs.append(model)
    for (name, p), (_, q) in zip(runs[1].module.named_parameters(), runs[0].module.named_parameters()):
        assert torch.equal(p, q), f"[rank {rank}] deferred + torch AdamW differs at {name}"
    # Direct gradient readers wait explicitly.
    model = runs[1]
    model.zero_grad()
    model(ids.chunk(world)[rank], tgt.chunk(world)[rank])[1].backward()
    ddp_mod.wait_all_deferred()
    norm = torch.nn.utils.clip_grad_norm_(model.parameters(), 1e9)
    ref = runs[0]
    ref.zero_grad()
    ref(ids.chunk(world)[rank], tgt.chunk(world)[rank])[1].backward()
    want = torch.nn.utils.clip_grad_norm_(ref.parameters(), 1e9)
    assert torch.equal(norm, want), (norm, want)


def test_ddp_deferred_buckets_with_a_plain_optimizer():
    run_distributed(_deferred_with_torch_adamw, 2)


@pytest.mark.parametrize("world", [2, 4])
def test_ddp_matches_full_batch_gradient(world):
    run_distributed(_default, world)


def test_ddp_with_one_bucket_per_parameter():
    run_distributed(_per_param_buckets, 2)


def test_ddp_with_a_single_bucket():
    run_distributed(_single_bucket, 2)


def test_ddp_without_backward_overlap():
    run_distributed(_no_overlap, 2)


def test_ddp_gradient_accumulation_under_no_sync():
    run_distributed(_accumulate, 2)


def test_ddp_bucket_layout():
    run_distributed(_layout, 2)
