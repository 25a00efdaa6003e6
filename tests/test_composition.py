"""The strategies compose: each 2x2 mesh equals the same model with one axis removed."""

from __future__ import annotations

import torch
import torch.distributed as dist
from torch import nn

from minidist.ddp import DistributedDataParallel
from minidist.fsdp import FullyShardedDataParallel
from minidist.mesh import ParallelMesh
from minidist.models import GPT, Block, GPTConfig, build_pipeline_layers
from minidist.pipeline import PipelineStage, build_schedule, partition_layers
from minidist.tensor_parallel import vocab_parallel_cross_entropy

from .harness import assert_close, run_distributed

CFG = GPTConfig(vocab_size=64, block_size=16, n_layer=4, n_head=4, n_embd=32)
BATCH = 8


def _data():
    g = torch.Generator().manual_seed(7)
    return (torch.randint(0, CFG.vocab_size, (BATCH, CFG.block_size), generator=g),
            torch.randint(0, CFG.vocab_size, (BATCH, CFG.block_size), generator=g))


def _loss(mesh):
    start = mesh.tp_rank * (CFG.vocab_size // mesh.tp_size)
    return lambda z, t: vocab_parallel_cross_entropy(z, t, group=mesh.tp_group, vocab_start=start)


def _tp_pp(rank, world):
    mesh = ParallelMesh(tp_size=2, pp_size=2)
    ids, tgt = _data()
    layers = build_pipeline_layers(CFG, tp_group=mesh.tp_group)
    x = ids
    for layer in layers:
        x = layer(x)
    ref_loss = _loss(mesh)(x, tgt)
    ref_loss.backward()
    ref_grads = [[p.grad.clone() for p in l.parameters()] for l in layers]

    layers = build_pipeline_layers(CFG, tp_group=mesh.tp_group)
    mine = partition_layers(layers, 2, mesh.pp_rank)
    off = next(i for i, l in enumerate(layers) if l is mine[0])
    stage = PipelineStage(nn.Sequential(*mine), mesh, loss_fn=_loss(mesh) if mesh.is_last_stage else None)
    loss = build_schedule("1f1b", stage, mesh, 4).step(inputs=ids, targets=tgt)
    if mesh.is_last_stage:
        assert_close(loss, ref_loss.detach(), f"[rank {rank}] tp2xpp2 loss", tol=1e-5)
    for li, layer in enumerate(mine):
        for pi, (p, w) in enumerate(zip(layer.parameters(), ref_grads[off + li])):
            assert_close(p.grad, w, f"[rank {rank}] layer {off + li} param {pi}", tol=2e-5)


def _tp_dp(rank, world):
    mesh = ParallelMesh(tp_size=2, pp_size=1)
    assert mesh.dp_size == 2
    ids, tgt = _data()
    ref = GPT(CFG, tp_group=mesh.tp_group)
    ref(ids, tgt)[1].backward()
    model = DistributedDataParallel(GPT(CFG, tp_group=mesh.tp_group), process_group=mesh.dp_group)
    # TP peers see the same rows, DP peers different ones: index by dp_rank only.
    model(ids.chunk(2)[mesh.dp_rank], tgt.chunk(2)[mesh.dp_rank])[1].backward()
    for (name, p), (_, r) in zip(model.module.named_parameters(), ref.named_parameters()):
        assert_close(p.grad, r.grad, f"[rank {rank}] tp2xdp2 {name}", tol=2e-5)


def _tp_fsdp(rank, world):
    mesh = ParallelMesh(tp_size=2, pp_size=1)
    ids, tgt = _data()
    mine = ids.chunk(2)[mesh.dp_rank], tgt.chunk(2)[mesh.dp_rank]
    ddp = DistributedDataParallel(GPT(CFG, tp_group=mesh.tp_group), process_group=mesh.dp_group)
    dl = ddp(*mine)[1]
    dl.backward()
    fsdp = FullyShardedDataParallel(GPT(CFG, tp_group=mesh.tp_group), unit_types=(Block,),
                                    process_group=mesh.dp_group)
    fl = fsdp(*mine)[1]
    fl.backward()
    assert_close(fl, dl, f"[rank {rank}] loss", tol=1e-6)
    names = {id(p): n for n, p in fsdp.module.named_parameters()}
    want = {n: p.grad for n, p in ddp.module.named_parameters()}
    for u in fsdp._units:
        parts = [torch.empty_like(u.flat_shard.grad) for _ in range(mesh.dp_size)]
        dist.all_gather(parts, u.flat_shard.grad.contiguous(), group=mesh.dp_group)
        flat = torch.cat(parts)[: u.total_numel]
        off = 0
        for p, n, shape in zip(u.params, u.numels, u.shapes):
            assert_close(flat[off : off + n].view(shape), want[names[id(p)]], f"[rank {rank}] {names[id(p)]}", tol=1e-6)
            off += n


def test_tensor_and_pipeline_parallel():
    run_distributed(_tp_pp, 4)


def test_tensor_and_data_parallel():
    run_distributed(_tp_dp, 4)


def test_tensor_parallel_with_fsdp():
    run_distributed(_tp_fsdp, 4)
