"""Tensor-parallel reductions on the fused B200 path.

``all_reduce_`` sums a bf16 activation (or activation gradient) over the
tensor-parallel group — the reference's ``g`` forward and ``f`` backward
(tensor_parallel.py:134-172).  ``row_parallel_fwd`` is the row-parallel linear:
local GEMM on this rank's slice of the input features, reduction of the
partial sums, then bias and residual added once.

Both route through :mod:`minidist.parallel.collectives`: a one-shot peer-memory
all-reduce kernel over NVLink when every rank of the group is on this node
(symmetric buffers from :mod:`minidist.parallel.symm`), and NCCL otherwise.
"""

from __future__ import annotations

import torch

from .. import comm
from ..ops import gemm as G


def all_reduce_(t: torch.Tensor, group) -> torch.Tensor:
    from . import collectives

    return collectives.all_reduce_(t, group)


def row_parallel_fwd(x_local: torch.Tensor, w_local: torch.Tensor, bias: torch.Tensor | None,
                     resid: torch.Tensor | None, group) -> torch.Tensor:
    """``resid + all_reduce(x_local @ w_local^T) + bias`` in bf16."""
    from . import collectives

    return collectives.gemm_all_reduce(x_local, w_local, bias, resid, group)
