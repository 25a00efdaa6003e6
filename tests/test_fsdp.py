"""ZeRO-3 sharding changes where values live, never what they are."""

from __future__ import annotations

import pytest
import torch
import torch.distributed as dist

from minidist.ddp import DistributedDataParallel
from minidist.fsdp import FullyShardedDataParallel, MixedPrecisionPolicy
from minidist.models import GPT, Block, GPTConfig

from .harness import assert_close, run_distributed, solo_group

CFG = GPTConfig(vocab_size=64, block_size=16, n_layer=3, n_head=4, n_embd=32)
BATCH, STEPS = 8, 4


def _batches(n):
    g = torch.Generator().manual_seed(1234)
    for _ in range(n):
        yield (torch.randint(0, CFG.vocab_size, (BATCH, CFG.block_size), generator=g),
               torch.randint(0, CFG.vocab_size, (BATCH, CFG.block_size), generator=g))


def _full_grads_from_shards(model, world, group=None):
    names = {id(p): n for n, p in model.module.named_parameters()}
    out = {}
    for u in model._units:
        parts = [torch.empty_like(u.flat_shard.grad) for _ in range(world)]
        dist.all_gather(parts, u.flat_shard.grad.contiguous(), group=group)
        flat = torch.cat(parts)[: u.total_numel]
        off = 0
        for p, n, shape in zip(u.params, u.numels, u.shapes):
            out[names[id(p)]] = flat[off : off + n].view(shape)
            off += n
    return out


def _train(model, rank, world, steps=STEPS, lr=1e-2):
    # SGD keeps the FSDP-vs-DDP comparison meaningful: reduce-scatter and
    # all-reduce sum in different orders (~1e-7 relative), which Adam's
    # scale-free update would amplify on tiny gradients.
    opt = torch.optim.SGD(model.parameters(), lr=lr)
    losses = []
    for ids, tgt in _batches(steps):
        opt.zero_grad(set_to_none=True)
        loss = model(ids.chunk(world)[rank], tgt.chunk(world)[rank])[1]
        loss.backward()
        opt.step()
        losses.append(loss.item())
    return losses


def _grads_match(rank, world):
    solo = solo_group(rank, world)
    ids, tgt = next(_batches(1))
    mine = ids.chunk(world)[rank], tgt.chunk(world)[rank]
    ddp = DistributedDataParallel(GPT(CFG, tp_group=solo))
    dl = ddp(*mine)[1]
    dl.backward()
    fsdp = FullyShardedDataParallel(GPT(CFG, tp_group=solo), unit_types=(Block,))
    fl = fsdp(*mine)[1]
    fl.backward()
    assert_close(fl, dl, f"[rank {rank}] loss", tol=1e-6)
    got = _full_grads_from_shards(fsdp, world)
    for name, p in ddp.module.named_parameters():
        assert_close(got[name], p.grad, f"[rank {rank}] grad {name}", tol=1e-6)


def _weights_match(rank, world):
    solo = solo_group(rank, world)
    ddp = DistributedDataParallel(GPT(CFG, tp_group=solo))
    dl = _train(ddp, rank, world)
    fsdp = FullyShardedDataParallel(GPT(CFG, tp_group=solo), unit_types=(Block,))
    fl = _train(fsdp, rank, world)
    for s, (a, b) in enumerate(zip(dl, fl)):
        assert abs(a - b) < 1e-5, f"[rank {rank}] step {s}: fsdp {b} vs ddp {a}"
    with fsdp.summon_full_params():
        got = dict(fsdp.module.named_parameters())
        for name, p in ddp.module.named_parameters():
            assert_close(got[name], p, f"[rank {rank}] weight {name}", tol=1e-5)


def _shards(rank, world):
    solo = solo_group(rank, world)
    model = FullyShardedDataParallel(GPT(CFG, tp_group=solo), unit_types=(Block,))
    full = sum(p.numel() for p in GPT(CFG, tp_group=solo).parameters())
    local = sum(p.numel() for p in model.parameters())
    assert local < full and local <= 1.25 * full / world
    s = model.memory_summary()
    assert s["num_units"] == CFG.n_layer + 1
    assert s["fsdp_state_MB"] < s["ddp_state_MB"]


def _frees(rank, world):
    solo = solo_group(rank, world)
    model = FullyShardedDataParallel(GPT(CFG, tp_group=solo), unit_types=(Block,))
    ids, tgt = next(_batches(1))
    model(ids.chunk(world)[rank], tgt.chunk(world)[rank])[1].backward()
    for u in model._units:
        assert not u.is_unsharded, u.name
        assert u._full.untyped_storage().nbytes() == 0, f"{u.name} still holds gathered memory"
        assert all(p.grad is None for p in u.params), f"{u.name} kept a full-size gradient"


def _zero2(rank, world):
    solo = solo_group(rank, world)
    a = _train(FullyShardedDataParallel(GPT(CFG, tp_group=solo), unit_types=(Block,)), rank, world)
    b = _train(FullyShardedDataParallel(GPT(CFG, tp_group=solo), unit_types=(Block,),
                                        reshard_after_forward=False), rank, world)
    for s, (x, y) in enumerate(zip(a, b)):
        assert abs(x - y) < 1e-6, f"[rank {rank}] step {s}: ZeRO-2 {y} vs ZeRO-3 {x}"


def _bf16(rank, world):
    solo = solo_group(rank, world)
    ref = _train(FullyShardedDataParallel(GPT(CFG, tp_group=solo), unit_types=(Block,)), rank, world, steps=2)
    m = FullyShardedDataParallel(GPT(CFG, tp_group=solo), unit_types=(Block,),
                                 mixed_precision=MixedPrecisionPolicy(torch.bfloat16, torch.float32))
    got = _train(m, rank, world, steps=2)
    assert m._units[0].flat_shard.dtype == torch.float32
    for s, (a, b) in enumerate(zip(ref, got)):
        assert abs(a - b) < 0.05, f"[rank {rank}] step {s}: bf16 {b:.4f} vs fp32 {a:.4f}"


def _accumulate(rank, world):
    solo = solo_group(rank, world)
    ids, tgt = next(_batches(1))
    ids, tgt = ids.chunk(world)[rank], tgt.chunk(world)[rank]
    one = FullyShardedDataParallel(GPT(CFG, tp_group=solo), unit_types=(Block,))
    one(ids, tgt)[1].backward()
    want = [p.grad.clone() for p in one.parameters()]
    acc = FullyShardedDataParallel(GPT(CFG, tp_group=solo), unit_types=(Block,))
    with acc.no_sync():
        for i, t in zip(ids.chunk(2), tgt.chunk(2)):
            (acc(i, t)[1] / 2).backward()
    acc.finish_gradient_sync()
    for k, (g, w) in enumerate(zip(acc.parameters(), want)):
        assert_close(g.grad, w, f"[rank {rank}] shard grad {k}", tol=2e-5)


@pytest.mark.parametrize("world", [2, 4])
def test_fsdp_gradients_match_ddp(world):
    run_distributed(_grads_match, world)


@pytest.mark.parametrize("world", [2, 4])
def test_fsdp_matches_ddp(world):
    run_distributed(_weights_match, world)


@pytest.mark.parametrize("world", [2, 4])
def test_fsdp_actually_shards(world):
    run_distributed(_shards, world)


def _casts_invalidated(rank, world):
    """Every gather marks the cached low-precision casts of the unit's parameters stale (the
    gathered bytes change without the parameters' version counters moving)."""
    solo = solo_group(rank, world)
    model = FullyShardedDataParallel(GPT(CFG, tp_group=solo), unit_types=(Block,))
    for u in model._units:
        for p in u.params:
            p._md_bf16_ver = p._version  # as a cast made at this version would record
        u.reshard()
        u.unshard()
        assert all(p._md_bf16_ver is None for p in u.params), u.name
        u.reshard()


def test_fsdp_gather_invalidates_cached_casts():
    run_distributed(_casts_invalidated, 2)


def test_fsdp_frees_gathered_parameters():
    run_distributed(_frees, 2)


def test_fsdp_reshard_after_forward_is_transparent():
    run_distributed(_zero2, 2)


def test_fsdp_mixed_precision():
    run_distributed(_bf16, 2)


def test_fsdp_gradient_accumulation():
    run_distributed(_accumulate, 2)
