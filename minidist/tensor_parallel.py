r"""Megatron-style tensor parallelism: column/row-sharded linears, a vocabulary-
sharded embedding, and cross-entropy over vocabulary-sharded logits.

A column-parallel linear (output features split) followed by a row-parallel
linear (input features split) needs a single reduction at the end: the
elementwise op between them commutes with the column split (reference
tensor_parallel.py:1-36).  Two conjugate operators bracket every parallel
region:

* ``f`` (:func:`copy_to_tensor_parallel`): identity forward, all-reduce of the
  input gradient backward;
* ``g`` (:func:`reduce_from_tensor_parallel`): all-reduce forward, identity
  backward.

Weights are materialised in full from a seed and then sliced, so a ``tp=N``
model holds exactly the weights of the ``tp=1`` model (reference
tensor_parallel.py:82-99, 232-243).  That makes "TP reproduces the single-GPU
model" a testable statement and keeps checkpoints interchangeable.

This module is the portable path (Gloo/CPU and any CUDA model that is not
routed through the fused kernels).  On B200 the GPT model's tensor-parallel
reductions run in peer-memory kernels of :mod:`minidist.parallel.collectives`
(the ``g`` reduction fused into the row-parallel GEMM, the ``f`` reduction into
the data-gradient GEMM, the embedding's ``g`` replaced by a gather from the
owning rank's shard).
"""

from __future__ import annotations

import math

import torch
import torch.distributed as dist
import torch.nn.functional as F
from torch import nn

from . import comm

__all__ = [
    "ColumnParallelLinear",
    "RowParallelLinear",
    "VocabParallelEmbedding",
    "vocab_parallel_cross_entropy",
    "copy_to_tensor_parallel",
    "reduce_from_tensor_parallel",
    "gather_from_tensor_parallel",
    "scatter_to_tensor_parallel",
    "full_linear_weight",
    "full_embedding_weight",
]


# ---------------------------------------------------------------------------
# Deterministic full-weight construction.  The draws (CPU generator seeded
# with `seed`, uniform(-1/sqrt(fan_in), 1/sqrt(fan_in)) for linears,
# normal(0, 0.02) for embeddings, both in fp32) follow the reference
# (tensor_parallel.py:82-99) so that the same seed yields bit-identical
# weights in both frameworks.
# ---------------------------------------------------------------------------


def full_linear_weight(out_features: int, in_features: int, seed: int, dtype=torch.float32) -> torch.Tensor:
    gen = torch.Generator(device="cpu").manual_seed(seed)
    bound = 1.0 / math.sqrt(in_features)
    w = torch.empty(out_features, in_features, dtype=torch.float32).uniform_(-bound, bound, generator=gen)
    return w.to(dtype)


def full_embedding_weight(num_embeddings: int, dim: int, seed: int, dtype=torch.float32) -> torch.Tensor:
    gen = torch.Generator(device="cpu").manual_seed(seed)
    w = torch.empty(num_embeddings, dim, dtype=torch.float32).normal_(0.0, 0.02, generator=gen)
    return w.to(dtype)


# ---------------------------------------------------------------------------
# Last-dimension split / gather
# ---------------------------------------------------------------------------


def _split_last(t: torch.Tensor, world: int, rank: int) -> torch.Tensor:
    n = t.size(-1)
    if n % world:
        raise ValueError(f"cannot split a last dimension of {n} over {world} ranks")
    step = n // world
    return t[..., rank * step : (rank + 1) * step].contiguous()


def _gather_last(t: torch.Tensor, group, world: int) -> torch.Tensor:
    if world == 1:
        return t
    t = t.contiguous()
    # One contiguous all-gather over a leading "rank" axis, then move that axis
    # next to the last dimension.
    out = torch.empty((world, *t.shape), dtype=t.dtype, device=t.device)
    comm.all_gather_into_tensor(out.view(-1), t.view(-1), group=group)
    return out.movedim(0, -2).reshape(*t.shape[:-1], world * t.shape[-1])


# ---------------------------------------------------------------------------
# f / g and the gather/scatter pair
# ---------------------------------------------------------------------------


class _CopyToTP(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, group):
        ctx.group = group
        return x

    @staticmethod
    def backward(ctx, grad):
        if comm.get_world_size(ctx.group) > 1:
            grad = grad.contiguous().clone()
            comm.all_reduce(grad, group=ctx.group)
        return grad, None


class _ReduceFromTP(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, group):
        if comm.get_world_size(group) > 1:
            x = x.contiguous().clone()
            comm.all_reduce(x, group=group)
        return x

    @staticmethod
    def backward(ctx, grad):
        return grad, None


class _GatherFromTP(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, group):
        ctx.world, ctx.rank = comm.get_world_size(group), comm.get_rank(group)
        return _gather_last(x, group, ctx.world)

    @staticmethod
    def backward(ctx, grad):
        return _split_last(grad, ctx.world, ctx.rank), None


class _ScatterToTP(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, group):
        ctx.group, ctx.world = group, comm.get_world_size(group)
        return _split_last(x, ctx.world, comm.get_rank(group))

    @staticmethod
    def backward(ctx, grad):
        return _gather_last(grad, ctx.group, ctx.world), None


def copy_to_tensor_parallel(x, group=None):
    """``f``: identity forward, all-reduce backward."""
    return _CopyToTP.apply(x, group)


def reduce_from_tensor_parallel(x, group=None):
    """``g``: all-reduce forward, identity backward."""
    return _ReduceFromTP.apply(x, group)


def gather_from_tensor_parallel(x, group=None):
    """All-gather along the last dimension forward; take this rank's slice backward."""
    return _GatherFromTP.apply(x, group)


def scatter_to_tensor_parallel(x, group=None):
    """Take this rank's slice of the last dimension forward; all-gather backward."""
    return _ScatterToTP.apply(x, group)


# ---------------------------------------------------------------------------
# Parallel layers
# ---------------------------------------------------------------------------


class _TPLinear(nn.Module):
    def __init__(self, group):
        super().__init__()
        self.group = group
        self.world = comm.get_world_size(group)
        self.rank = comm.get_rank(group)

    def _shard_of_full(self, out_f: int, in_f: int, dim: int, seed: int, device, dtype) -> torch.Tensor:
        full = full_linear_weight(out_f, in_f, seed)
        return full.chunk(self.world, dim=dim)[self.rank].contiguous().to(device=device, dtype=dtype)


class ColumnParallelLinear(_TPLinear):
    """``y = x A^T + b`` with ``A``'s output rows split across the group.

    Input replicated, output sharded on its last dimension (or gathered when
    ``gather_output=True``).
    """

    def __init__(self, in_features, out_features, bias=True, gather_output=False, group=None, seed=0,
                 device=None, dtype=None):
        super().__init__(group)
        if out_features % self.world:
            raise ValueError(f"out_features={out_features} not divisible by tp_size={self.world}")
        self.in_features, self.out_features = in_features, out_features
        self.out_features_per_partition = out_features // self.world
        self.gather_output = gather_output
        self.weight = nn.Parameter(self._shard_of_full(out_features, in_features, 0, seed, device, dtype))
        if bias:
            self.bias = nn.Parameter(torch.zeros(self.out_features_per_partition, device=device, dtype=dtype))
        else:
            self.register_parameter("bias", None)

    def forward(self, x):
        y = F.linear(copy_to_tensor_parallel(x, self.group), self.weight, self.bias)
        return gather_from_tensor_parallel(y, self.group) if self.gather_output else y

    @torch.no_grad()
    def set_full_weight(self, weight, bias=None):
        self.weight.copy_(weight.chunk(self.world, dim=0)[self.rank])
        if bias is not None and self.bias is not None:
            self.bias.copy_(bias.chunk(self.world, dim=0)[self.rank])

    def extra_repr(self):
        return (f"in={self.in_features}, out={self.out_features} "
                f"(local {self.out_features_per_partition}), tp={self.world}")


class RowParallelLinear(_TPLinear):
    """``y = x A^T + b`` with ``A``'s input columns split; partial sums are reduced by ``g``.

    The bias is replicated and added after the reduction (adding it before
    would count it ``world`` times).
    """

    def __init__(self, in_features, out_features, bias=True, input_is_parallel=True, group=None, seed=0,
                 device=None, dtype=None):
        super().__init__(group)
        if in_features % self.world:
            raise ValueError(f"in_features={in_features} not divisible by tp_size={self.world}")
        self.in_features, self.out_features = in_features, out_features
        self.in_features_per_partition = in_features // self.world
        self.input_is_parallel = input_is_parallel
        self.weight = nn.Parameter(self._shard_of_full(out_features, in_features, 1, seed, device, dtype))
        if bias:
            self.bias = nn.Parameter(torch.zeros(out_features, device=device, dtype=dtype))
        else:
            self.register_parameter("bias", None)

    def forward(self, x):
        if not self.input_is_parallel:
            x = scatter_to_tensor_parallel(x, self.group)
        y = reduce_from_tensor_parallel(F.linear(x, self.weight), self.group)
        return y + self.bias if self.bias is not None else y

    @torch.no_grad()
    def set_full_weight(self, weight, bias=None):
        self.weight.copy_(weight.chunk(self.world, dim=1)[self.rank])
        if bias is not None and self.bias is not None:
            self.bias.copy_(bias)

    def extra_repr(self):
        return (f"in={self.in_features} (local {self.in_features_per_partition}), "
                f"out={self.out_features}, tp={self.world}")


class VocabParallelEmbedding(nn.Module):
    """Embedding table split by contiguous vocabulary ranges; ``g`` assembles the rows."""

    def __init__(self, num_embeddings, embedding_dim, group=None, seed=0, device=None, dtype=None):
        super().__init__()
        self.group = group
        self.world = comm.get_world_size(group)
        self.rank = comm.get_rank(group)
        if num_embeddings % self.world:
            raise ValueError(f"vocab size {num_embeddings} not divisible by tp_size={self.world}")
        self.num_embeddings, self.embedding_dim = num_embeddings, embedding_dim
        self.num_embeddings_per_partition = num_embeddings // self.world
        self.vocab_start = self.rank * self.num_embeddings_per_partition
        self.vocab_end = self.vocab_start + self.num_embeddings_per_partition
        full = full_embedding_weight(num_embeddings, embedding_dim, seed)
        self.weight = nn.Parameter(full[self.vocab_start : self.vocab_end].contiguous().to(device=device, dtype=dtype))

    def forward(self, input_ids):
        if self.world == 1:
            return F.embedding(input_ids, self.weight)
        outside = (input_ids < self.vocab_start) | (input_ids >= self.vocab_end)
        local = (input_ids - self.vocab_start).clamp(0, self.num_embeddings_per_partition - 1)
        rows = F.embedding(local, self.weight).masked_fill(outside.unsqueeze(-1), 0.0)
        return reduce_from_tensor_parallel(rows, self.group)

    @torch.no_grad()
    def set_full_weight(self, weight):
        self.weight.copy_(weight[self.vocab_start : self.vocab_end])


# ---------------------------------------------------------------------------
# Cross-entropy over vocabulary-sharded logits
# ---------------------------------------------------------------------------


class _ShardedCrossEntropy(torch.autograd.Function):
    """Per-token ``logsumexp(z) - z_target`` where each rank holds ``z[:, shard]``.

    log-sum-exp decomposes over a partition of the vocabulary into three
    per-token reductions — a MAX of the shard maxima, a SUM of the rescaled
    exp-sums, and a SUM that delivers the target logit from the rank owning
    it — so the ``[tokens, V]`` logits never cross the interconnect (reference
    tensor_parallel.py:428-492).  The backward ``softmax - onehot`` is local.
    """

    @staticmethod
    def forward(ctx, logits, target, group, vocab_start):
        z = logits.float()
        width = z.size(-1)
        world = comm.get_world_size(group)
        zmax = z.amax(dim=-1)
        if world > 1:
            dist.all_reduce(zmax, op=dist.ReduceOp.MAX, group=group)
        shifted = z - zmax.unsqueeze(-1)
        e = shifted.exp()
        sumexp = e.sum(dim=-1)
        if world > 1:
            dist.all_reduce(sumexp, op=dist.ReduceOp.SUM, group=group)
        owned = (target >= vocab_start) & (target < vocab_start + width)
        local_t = (target - vocab_start).clamp(0, width - 1)
        picked = shifted.gather(-1, local_t.unsqueeze(-1)).squeeze(-1) * owned
        if world > 1:
            dist.all_reduce(picked, op=dist.ReduceOp.SUM, group=group)
        loss = sumexp.log() - picked
        ctx.save_for_backward(e.div_(sumexp.unsqueeze(-1)), owned, local_t)
        ctx.in_dtype = logits.dtype
        return loss

    @staticmethod
    def backward(ctx, grad_loss):
        probs, owned, local_t = ctx.saved_tensors
        g = probs
        g.scatter_add_(-1, local_t.unsqueeze(-1), -owned.to(g.dtype).unsqueeze(-1))
        g.mul_(grad_loss.unsqueeze(-1))
        return g.to(ctx.in_dtype), None, None, None


def vocab_parallel_cross_entropy(logits, target, group=None, vocab_start: int = 0, reduction: str = "mean"):
    """Cross entropy of vocabulary-sharded ``logits [..., V/tp]`` against global ids ``target``."""
    flat = logits.reshape(-1, logits.size(-1))
    loss = _ShardedCrossEntropy.apply(flat, target.reshape(-1), group, vocab_start)
    if reduction == "mean":
        return loss.mean()
    if reduction == "sum":
        return loss.sum()
    if reduction == "none":
        return loss.view(target.shape)
    raise ValueError(f"unknown reduction {reduction!r}")
