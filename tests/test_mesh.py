"""Mesh coordinates: rank <-> (pp, dp, tp), contiguous TP groups, strided PP groups."""

from __future__ import annotations

import pytest
import torch.distributed as dist

from minidist.mesh import ParallelMesh

from .harness import run_distributed


def _roundtrip(rank, world, tp, pp):
    mesh = ParallelMesh(tp_size=tp, pp_size=pp)
    assert mesh.tp_size * mesh.dp_size * mesh.pp_size == world
    seen = set()
    for r in range(world):
        c = mesh.coord_of(r)
        assert mesh.rank_of(c.pp, c.dp, c.tp) == r
        seen.add((c.pp, c.dp, c.tp))
    assert len(seen) == world
    assert dist.get_world_size(mesh.tp_group) == tp
    assert dist.get_world_size(mesh.pp_group) == pp
    assert dist.get_world_size(mesh.dp_group) == world // (tp * pp)


def _layout(rank, world, tp, pp):
    mesh = ParallelMesh(tp_size=tp, pp_size=pp)
    tp_members = mesh.axis_ranks("tp")
    assert tp_members == list(range(tp_members[0], tp_members[0] + tp)), f"TP group {tp_members} not contiguous"
    stride = mesh.dp_size * mesh.tp_size
    assert mesh.pp_ranks == sorted(mesh.pp_ranks)
    assert all(b - a == stride for a, b in zip(mesh.pp_ranks, mesh.pp_ranks[1:]))


def _stage_flags(rank, world, tp, pp):
    mesh = ParallelMesh(tp_size=tp, pp_size=pp)
    assert mesh.is_first_stage == (mesh.pp_rank == 0)
    assert mesh.is_last_stage == (mesh.pp_rank == pp - 1)
    assert (mesh.prev_stage_rank is None) == mesh.is_first_stage
    assert (mesh.next_stage_rank is None) == mesh.is_last_stage
    if not mesh.is_last_stage:
        assert mesh.coord_of(mesh.next_stage_rank).pp == mesh.pp_rank + 1


def _bad_factorisation(rank, world):
    with pytest.raises(ValueError):
        ParallelMesh(tp_size=3, pp_size=1)


@pytest.mark.parametrize("tp,pp", [(1, 1), (2, 1), (1, 2), (2, 2), (4, 1), (1, 4)])
def test_mesh_coordinate_roundtrip(tp, pp):
    run_distributed(_roundtrip, 4, tp, pp)


@pytest.mark.parametrize("tp,pp", [(2, 2), (2, 1), (1, 2)])
def test_tensor_parallel_groups_are_contiguous(tp, pp):
    run_distributed(_layout, 4, tp, pp)


@pytest.mark.parametrize("tp,pp", [(2, 2), (1, 4)])
def test_pipeline_stage_flags(tp, pp):
    run_distributed(_stage_flags, 4, tp, pp)


def test_invalid_factorisation_is_rejected():
    run_distributed(_bad_factorisation, 2)
