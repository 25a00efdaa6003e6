"""Collectives used by the fused path (NCCL baseline; peer-memory kernels added later)."""

from __future__ import annotations

import torch

from .. import comm
from ..ops import gemm as G


def make_bucket_reducer(ddp, required: bool = False):
    return None


def all_reduce_(t: torch.Tensor, group) -> torch.Tensor:
    comm.all_reduce(t, group=group)
    return t


def gemm_all_reduce(x_local, w_local, bias, resid, group):
    out = G.linear_fwd(x_local, w_local)
    comm.all_reduce(out, group=group)
    acc = out.float()
    if bias is not None:
        acc += bias
    if resid is not None:
        acc += resid.float()
    res = G.empty_padded(out.shape[0], out.shape[1], device=out.device)
    res.copy_(acc)
    return res
