r"""The 3-D (pipeline x data x tensor) process mesh.

Flat ranks map to coordinates with tensor parallelism varying fastest::

    rank = pp * (dp_size * tp_size) + dp * tp_size + tp

so a tensor-parallel group is a block of consecutive ranks (the GPUs of one
NVSwitch domain under torchrun), data-parallel peers sit ``tp_size`` apart and
pipeline neighbours ``dp_size * tp_size`` apart (reference mesh.py:1-33,
104-116).  On one 8xB200 box every pair of GPUs has the same NVSwitch
bandwidth, but the ordering still matters across boxes and keeps the layout
identical to the reference's, which checkpoints and launch scripts rely on.

Besides the process groups, the mesh hands out the per-axis native
communicators used by the fused NVLink kernels
(:func:`minidist.parallel.symm.communicator`), built lazily on first use.
"""

from __future__ import annotations

from dataclasses import dataclass

import torch
import torch.distributed as dist

from .comm import current_device, get_rank, get_world_size

__all__ = ["ParallelMesh", "torch_dtype_bytes"]


@dataclass(frozen=True)
class _Coord:
    pp: int
    dp: int
    tp: int


class ParallelMesh:
    """Factorise the world into ``(pp, dp, tp)`` axes and build every subgroup.

    ``dp_size`` defaults to ``world // (tp_size * pp_size)``; an inconsistent
    factorisation raises ``ValueError``.  ``dist.new_group`` is collective, so
    every rank creates every group in the same order — TP groups, then DP
    groups, then PP groups — even the ones it is not a member of.
    """

    def __init__(self, tp_size: int = 1, pp_size: int = 1, dp_size: int | None = None):
        world = get_world_size()
        if min(tp_size, pp_size) < 1:
            raise ValueError("parallel degrees must be >= 1")
        if dp_size is None:
            dp_size = world // (tp_size * pp_size)
        if dp_size < 1 or tp_size * pp_size * dp_size != world:
            raise ValueError(
                f"tp({tp_size}) * pp({pp_size}) * dp({dp_size}) = {tp_size * pp_size * dp_size} "
                f"!= world_size({world})"
            )
        self.tp_size, self.pp_size, self.dp_size = tp_size, pp_size, dp_size
        self.world_size = world
        self.rank = get_rank()
        self.device = current_device()
        c = self.coord_of(self.rank)
        self.pp_rank, self.dp_rank, self.tp_rank = c.pp, c.dp, c.tp

        self._groups: dict[str, dist.ProcessGroup | None] = {"tp": None, "dp": None, "pp": None}
        self._members: dict[str, list[int]] = {
            "tp": [self.rank_of(self.pp_rank, self.dp_rank, t) for t in range(tp_size)],
            "dp": [self.rank_of(self.pp_rank, d, self.tp_rank) for d in range(dp_size)],
            "pp": [self.rank_of(p, self.dp_rank, self.tp_rank) for p in range(pp_size)],
        }
        self.pp_ranks: list[int] = list(self._members["pp"]) if world > 1 else [self.rank]
        if dist.is_available() and dist.is_initialized() and world > 1:
            self._build_groups()

    # -- coordinate algebra -------------------------------------------------

    def coord_of(self, rank: int) -> _Coord:
        tp = rank % self.tp_size
        rest = rank // self.tp_size
        return _Coord(pp=rest // self.dp_size, dp=rest % self.dp_size, tp=tp)

    def rank_of(self, pp: int, dp: int, tp: int) -> int:
        return (pp * self.dp_size + dp) * self.tp_size + tp

    # -- groups -------------------------------------------------------------

    def _axis_rank_lists(self, axis: str) -> list[list[int]]:
        P, D, T = self.pp_size, self.dp_size, self.tp_size
        if axis == "tp":
            return [[self.rank_of(p, d, t) for t in range(T)] for p in range(P) for d in range(D)]
        if axis == "dp":
            return [[self.rank_of(p, d, t) for d in range(D)] for p in range(P) for t in range(T)]
        return [[self.rank_of(p, d, t) for p in range(P)] for d in range(D) for t in range(T)]

    def _build_groups(self) -> None:
        for axis in ("tp", "dp", "pp"):
            for ranks in self._axis_rank_lists(axis):
                g = dist.new_group(ranks)
                if self.rank in ranks:
                    self._groups[axis] = g
        # A second pipeline group carries the backward (gradient) traffic, so on
        # NCCL the two directions run on separate communicator streams: a send of
        # the next activation can then never sit in front of the receive of the
        # current gradient.  Created after every reference group, so the order of
        # the groups above is unchanged.
        self._groups["pp_grad"] = self._groups["pp"]
        if self.pp_size > 1:
            for ranks in self._axis_rank_lists("pp"):
                g = dist.new_group(ranks)
                if self.rank in ranks:
                    self._groups["pp_grad"] = g

    def axis_ranks(self, axis: str) -> list[int]:
        """Global ranks of this rank's group along ``axis`` ("tp", "dp" or "pp"), in axis order."""
        return list(self._members[axis])

    @property
    def tp_group(self):
        return self._groups["tp"]

    @property
    def dp_group(self):
        return self._groups["dp"]

    @property
    def pp_group(self):
        return self._groups["pp"]

    @property
    def pp_grad_group(self):
        """Same ranks as :attr:`pp_group`; the pipeline sends gradients on it."""
        return self._groups["pp_grad"]

    @property
    def is_first_stage(self) -> bool:
        return self.pp_rank == 0

    @property
    def is_last_stage(self) -> bool:
        return self.pp_rank == self.pp_size - 1

    @property
    def prev_stage_rank(self) -> int | None:
        return None if self.is_first_stage else self.pp_ranks[self.pp_rank - 1]

    @property
    def next_stage_rank(self) -> int | None:
        return None if self.is_last_stage else self.pp_ranks[self.pp_rank + 1]

    def communicator(self, axis: str):
        """Native peer-memory communicator over ``axis`` (CUDA + NCCL runs only)."""
        from .parallel import symm

        return symm.communicator(self._groups[axis], self.axis_ranks(axis))

    def describe(self) -> str:
        return (
            f"world={self.world_size}  tp={self.tp_size} dp={self.dp_size} pp={self.pp_size}  |  "
            f"rank {self.rank} -> (pp={self.pp_rank}, dp={self.dp_rank}, tp={self.tp_rank})"
        )

    def __repr__(self) -> str:  # pragma: no cover
        return f"ParallelMesh({self.describe()})"


def torch_dtype_bytes(dtype: torch.dtype) -> int:
    """Bytes per element of ``dtype``."""
    return dtype.itemsize
