"""Tensor parallelism reproduces the unsharded computation."""

from __future__ import annotations

import pytest
import torch
import torch.nn.functional as F

from minidist.models import GPT, GPTConfig
from minidist.tensor_parallel import (
    ColumnParallelLinear,
    RowParallelLinear,
    VocabParallelEmbedding,
    full_embedding_weight,
    full_linear_weight,
    gather_from_tensor_parallel,
    vocab_parallel_cross_entropy,
)

from .harness import all_ranks_agree, assert_close, run_distributed, solo_group

CFG = GPTConfig(vocab_size=64, block_size=16, n_layer=2, n_head=4, n_embd=32)


def _column(rank, world):
    layer = ColumnParallelLinear(16, 32, bias=True, seed=7)
    x = torch.randn(4, 16, requires_grad=True)
    y = gather_from_tensor_parallel(layer(x), None)
    w = full_linear_weight(32, 16, 7)
    assert_close(y, F.linear(x, w), f"[rank {rank}] column forward")
    y.sum().backward()
    # Only correct if `f` all-reduces the partial input gradients.
    assert_close(x.grad, w.sum(0).expand(4, 16), f"[rank {rank}] column input grad", tol=1e-4)


def _row(rank, world):
    layer = RowParallelLinear(32, 16, bias=True, input_is_parallel=False, seed=11)
    x = torch.randn(4, 32)
    assert_close(layer(x), F.linear(x, full_linear_weight(16, 32, 11)), f"[rank {rank}] row forward")


def _embedding(rank, world):
    emb = VocabParallelEmbedding(32, 8, seed=3)
    ids = torch.randint(0, 32, (3, 5))
    assert_close(emb(ids), F.embedding(ids, full_embedding_weight(32, 8, 3)), f"[rank {rank}] embedding")


def _cross_entropy(rank, world):
    n, vocab = 12, 32
    shard = vocab // world
    lo = rank * shard
    logits = torch.randn(n, vocab, generator=torch.Generator().manual_seed(5))
    tgt = torch.randint(0, vocab, (n,), generator=torch.Generator().manual_seed(6))
    local = logits[:, lo : lo + shard].clone().requires_grad_(True)
    loss = vocab_parallel_cross_entropy(local, tgt, group=None, vocab_start=lo)
    ref_in = logits.clone().requires_grad_(True)
    ref = F.cross_entropy(ref_in, tgt)
    assert_close(loss, ref, f"[rank {rank}] CE value")
    loss.backward()
    ref.backward()
    assert_close(local.grad, ref_in.grad[:, lo : lo + shard], f"[rank {rank}] CE grad")


def _gpt(rank, world):
    solo = solo_group(rank, world)
    sharded, ref = GPT(CFG, tp_group=None), GPT(CFG, tp_group=solo)
    ids = torch.randint(0, CFG.vocab_size, (2, CFG.block_size))
    tgt = torch.randint(0, CFG.vocab_size, (2, CFG.block_size))
    loss, ref_loss = sharded(ids, tgt)[1], ref(ids, tgt)[1]
    assert_close(loss, ref_loss, f"[rank {rank}] tp={world} loss", tol=1e-5)
    loss.backward()
    ref_loss.backward()
    assert_close(sharded.blocks[0].attn.qkv.weight.grad, ref.blocks[0].attn.qkv.weight.grad.chunk(world, 0)[rank],
                 f"[rank {rank}] qkv grad shard", tol=1e-4)
    assert_close(sharded.blocks[0].attn.proj.weight.grad,
                 ref.blocks[0].attn.proj.weight.grad.chunk(world, 1)[rank], f"[rank {rank}] proj grad shard", tol=1e-4)


def _replicated(rank, world):
    model = GPT(CFG, tp_group=None)
    ids = torch.randint(0, CFG.vocab_size, (2, CFG.block_size))
    tgt = torch.randint(0, CFG.vocab_size, (2, CFG.block_size))
    model(ids, tgt)[1].backward()
    for name, p in {
        "blocks.0.ln1.weight": model.blocks[0].ln1.weight,
        "blocks.0.ln2.bias": model.blocks[0].ln2.bias,
        "lm_head.ln_f.weight": model.lm_head.ln_f.weight,
        "blocks.0.attn.proj.bias": model.blocks[0].attn.proj.bias,
        "blocks.0.mlp.proj.bias": model.blocks[0].mlp.proj.bias,
    }.items():
        assert p.grad is not None, name
        assert all_ranks_agree(p.grad), f"[rank {rank}] replicated {name} has a rank-dependent gradient"


@pytest.mark.parametrize("world", [2, 4])
def test_column_parallel_linear(world):
    run_distributed(_column, world)


@pytest.mark.parametrize("world", [2, 4])
def test_row_parallel_linear(world):
    run_distributed(_row, world)


def test_vocab_parallel_embedding():
    run_distributed(_embedding, 2)


@pytest.mark.parametrize("world", [2, 4])
def test_vocab_parallel_cross_entropy(world):
    run_distributed(_cross_entropy, world)


@pytest.mark.parametrize("world", [2, 4])
def test_gpt_tensor_parallel_matches_single_device(world):
    run_distributed(_gpt, world)


def test_replicated_parameters_get_identical_gradients():
    run_distributed(_replicated, 2)
