"""GPipe and 1F1B reproduce the non-pipelined loss and gradients."""

from __future__ import annotations

import pytest
import torch
from torch import nn

from minidist.mesh import ParallelMesh
from minidist.models import GPTConfig, build_pipeline_layers
from minidist.pipeline import PipelineStage, build_schedule, partition_layers, theoretical_bubble_fraction
from minidist.tensor_parallel import vocab_parallel_cross_entropy

from .harness import assert_close, run_distributed

CFG = GPTConfig(vocab_size=64, block_size=16, n_layer=4, n_head=4, n_embd=32)
BATCH = 8


def _data():
    g = torch.Generator().manual_seed(99)
    return (torch.randint(0, CFG.vocab_size, (BATCH, CFG.block_size), generator=g),
            torch.randint(0, CFG.vocab_size, (BATCH, CFG.block_size), generator=g))


def _loss(group):
    return lambda logits, t: vocab_parallel_cross_entropy(logits, t, group=group, vocab_start=0)


def _stage(mesh, world):
    layers = build_pipeline_layers(CFG, tp_group=mesh.tp_group)
    mine = partition_layers(layers, world, mesh.pp_rank)
    offset = next(i for i, layer in enumerate(layers) if layer is mine[0])
    stage = PipelineStage(nn.Sequential(*mine), mesh, loss_fn=_loss(mesh.tp_group) if mesh.is_last_stage else None)
    return stage, mine, offset


def _reference(mesh, ids, tgt):
    layers = build_pipeline_layers(CFG, tp_group=mesh.tp_group)
    x = ids
    for layer in layers:
        x = layer(x)
    loss = _loss(mesh.tp_group)(x, tgt)
    loss.backward()
    return loss.detach(), [[p.grad.clone() if p.grad is not None else None for p in l.parameters()] for l in layers]


def _run(rank, world, name, m):
    mesh = ParallelMesh(tp_size=1, pp_size=world)
    ids, tgt = _data()
    ref_loss, ref_grads = _reference(mesh, ids, tgt)
    stage, mine, off = _stage(mesh, world)
    loss = build_schedule(name, stage, mesh, m).step(inputs=ids, targets=tgt)
    if mesh.is_last_stage:
        assert_close(loss, ref_loss, f"[rank {rank}] {name} loss", tol=1e-5)
    for li, layer in enumerate(mine):
        for pi, (p, want) in enumerate(zip(layer.parameters(), ref_grads[off + li])):
            assert p.grad is not None, f"[rank {rank}] layer {off + li} param {pi} has no grad"
            assert_close(p.grad, want, f"[rank {rank}] {name} layer {off + li} param {pi}", tol=2e-5)


def _gpipe(rank, world):
    _run(rank, world, "gpipe", 4)


def _onefoneb(rank, world):
    _run(rank, world, "1f1b", 4)


def _single_mb(rank, world):
    _run(rank, world, "1f1b", 1)


def _agree(rank, world):
    mesh = ParallelMesh(tp_size=1, pp_size=world)
    ids, tgt = _data()
    out = {}
    for name in ("gpipe", "1f1b"):
        stage, _, _ = _stage(mesh, world)
        sched = build_schedule(name, stage, mesh, 4)
        loss = sched.step(inputs=ids, targets=tgt)
        out[name] = (loss, [p.grad.clone() for p in stage.parameters()], sched.max_activations_in_flight)
    if mesh.is_last_stage:
        assert_close(out["1f1b"][0], out["gpipe"][0], f"[rank {rank}] loss", tol=1e-6)
    for i, (a, b) in enumerate(zip(out["gpipe"][1], out["1f1b"][1])):
        assert_close(b, a, f"[rank {rank}] grad {i}", tol=1e-6)
    assert out["1f1b"][2] <= out["gpipe"][2], "1F1B must not hold more activations than GPipe"


def _bubble(rank, world):
    mesh = ParallelMesh(tp_size=1, pp_size=world)
    ids, tgt = _data()
    reports = {}
    for m in (1, 4):
        stage, _, _ = _stage(mesh, world)
        sched = build_schedule("1f1b", stage, mesh, m)
        sched.step(inputs=ids, targets=tgt)
        reports[m] = sched.report()
    for m, r in reports.items():
        assert r["theoretical_bubble"] == pytest.approx(theoretical_bubble_fraction(world, m))
        assert 0.0 <= r["measured_bubble"] <= 1.0 and r["busy_s"] > 0.0
    if not mesh.is_first_stage:
        assert reports[1]["measured_bubble"] > 0.0


def _cover(rank, world):
    layers = [nn.Linear(2, 2) for _ in range(7)]
    got = [l for s in range(world) for l in partition_layers(layers, world, s)]
    assert got == layers


@pytest.mark.parametrize("world", [2, 4])
def test_gpipe_matches_single_process(world):
    run_distributed(_gpipe, world)


@pytest.mark.parametrize("world", [2, 4])
def test_1f1b_matches_single_process(world):
    run_distributed(_onefoneb, world)


def test_single_microbatch():
    run_distributed(_single_mb, 2)


@pytest.mark.parametrize("world", [2, 4])
def test_schedules_agree(world):
    run_distributed(_agree, world)


@pytest.mark.parametrize("world", [2, 4])
def test_bubble_measurement(world):
    run_distributed(_bubble, world)


def test_layer_partitioning_is_a_cover():
    run_distributed(_cover, 3)
