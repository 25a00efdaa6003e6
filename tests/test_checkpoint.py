"""Checkpoints round-trip and consolidate into the unwrapped GPT format."""

from __future__ import annotations

import tempfile

import torch
from torch import nn

from minidist.ddp import DistributedDataParallel
from minidist.fsdp import FullyShardedDataParallel
from minidist.mesh import ParallelMesh
from minidist.models import GPT, Block, GPTConfig, build_pipeline_layers
from minidist.pipeline import partition_layers
from minidist.utils import checkpoint

from .harness import assert_close, run_distributed, solo_group

CFG = GPTConfig(vocab_size=64, block_size=16, n_layer=4, n_head=4, n_embd=32)


def test_single_process_roundtrip():
    model = GPT(CFG)
    with torch.no_grad():
        for p in model.parameters():
            p.add_(0.01)
    with tempfile.TemporaryDirectory() as d:
        checkpoint.save(d, model, step=3)
        fresh = GPT(CFG)
        manifest = checkpoint.load(d, fresh)
        assert manifest["step"] == 3
        for (n, a), (_, b) in zip(model.named_parameters(), fresh.named_parameters()):
            assert torch.equal(a, b), n
        merged = checkpoint.consolidate(d)
        assert set(merged) == set(model.state_dict())


def _tp_pp_consolidate(rank, world, d):
    mesh = ParallelMesh(tp_size=2, pp_size=2)
    layers = build_pipeline_layers(CFG, tp_group=mesh.tp_group)
    mine = nn.Sequential(*partition_layers(layers, 2, mesh.pp_rank))
    checkpoint.save(d, mine, mesh=mesh, step=1)
    g0 = solo_group_or_none()
    if rank == 0:
        merged = checkpoint.consolidate(d)
        ref = GPT(CFG, tp_group=g0).state_dict()
        assert set(merged) == set(ref), sorted(set(merged) ^ set(ref))
        for k in ref:
            assert torch.equal(merged[k], ref[k]), k


def solo_group_or_none():
    import torch.distributed as dist

    # new_group is collective: every rank creates it, only rank 0 is a member
    g = dist.new_group([0])
    return g if dist.get_rank() == 0 else None


def _fsdp_roundtrip(rank, world, d):
    solo = solo_group(rank, world)
    fsdp = FullyShardedDataParallel(GPT(CFG, tp_group=solo), unit_types=(Block,))
    with torch.no_grad():
        for p in fsdp.parameters():
            p.mul_(1.5)
    checkpoint.save(d, fsdp, step=2)
    fresh = FullyShardedDataParallel(GPT(CFG, tp_group=solo), unit_types=(Block,))
    checkpoint.load(d, fresh)
    for a, b in zip(fsdp.parameters(), fresh.parameters()):
        assert torch.equal(a, b)
    merged = checkpoint.consolidate(d)
    with fsdp.summon_full_params():  # collective: every rank enters
        for n, p in fsdp.module.named_parameters():
            assert_close(merged[n], p, n, tol=0)
    ddp = DistributedDataParallel(GPT(CFG, tp_group=solo))
    checkpoint.load(d, ddp)
    with fsdp.summon_full_params():
        for (n, a), (_, b) in zip(fsdp.module.named_parameters(), ddp.module.named_parameters()):
            assert torch.equal(a, b), n


def _tmp_dir(rank, world, fn):
    import torch.distributed as dist

    obj = [tempfile.mkdtemp() if rank == 0 else None]
    dist.broadcast_object_list(obj, src=0)
    fn(rank, world, obj[0])


def _tp_pp_body(rank, world):
    _tmp_dir(rank, world, _tp_pp_consolidate)


def _fsdp_body(rank, world):
    _tmp_dir(rank, world, _fsdp_roundtrip)


def test_tensor_pipeline_checkpoint_consolidates_to_gpt_format():
    run_distributed(_tp_pp_body, 4)


def test_fsdp_checkpoint_roundtrip_and_interop_with_ddp():
    run_distributed(_fsdp_body, 2)
