"""GPT decoder that tensor parallelism can shard and pipeline parallelism can split.

Architecture and parameter layout follow the reference (models/gpt.py:48-263)
so checkpoints are interchangeable: pre-LayerNorm blocks (eps 1e-5), learned
positions, GELU(tanh) MLP of width ``4*n_embd``, an *untied* LM head, and a QKV
projection whose output rows are interleaved per head as ``[n_head, 3,
head_dim]`` so that any contiguous column-parallel slice holds whole heads with
their own q, k and v (reference gpt.py:92-99).  Parameter names:
``embedding.wte.weight``, ``embedding.wpe``, ``blocks.{i}.{ln1,attn.qkv,
attn.proj,ln2,mlp.fc,mlp.proj}.*``, ``lm_head.{ln_f,head}.*``.

Two execution paths share those parameters:

* the portable path — plain modules (``F.linear``, SDPA, ``nn.LayerNorm``),
  used on CPU/Gloo and for fp32 runs;
* the fused B200 path (:mod:`minidist.models.fused_gpt`) — taken on CUDA when
  the step runs under bf16 autocast (``--precision bf16``) and the native
  library is present.  Each block is one autograd node that calls the
  hand-written sm_100a kernels: tcgen05 GEMMs with bias/GELU/residual
  epilogues, LayerNorm, flash attention, and a cross-entropy fused into the
  LM-head GEMM.  Weight gradients are written in place by the GEMM epilogues
  (see :mod:`minidist.ops.grads`).
"""

from __future__ import annotations

import os
from dataclasses import dataclass

import torch
import torch.nn.functional as F
from torch import nn

from .. import comm
from ..tensor_parallel import (
    ColumnParallelLinear,
    RowParallelLinear,
    VocabParallelEmbedding,
    vocab_parallel_cross_entropy,
)

__all__ = ["GPTConfig", "GPT", "Block", "Embedding", "LMHead", "build_pipeline_layers"]


@dataclass
class GPTConfig:
    vocab_size: int = 1024
    block_size: int = 128
    n_layer: int = 4
    n_head: int = 4
    n_embd: int = 128
    dropout: float = 0.0
    bias: bool = True
    seed: int = 1234

    @property
    def head_dim(self) -> int:
        return self.n_embd // self.n_head

    def param_count(self) -> int:
        """Parameters of the untied model (embeddings + blocks + final LN + head)."""
        n, v = self.n_embd, self.vocab_size
        per_block = 12 * n * n + 4 * n + (9 * n if self.bias else 0)
        return v * n + self.block_size * n + self.n_layer * per_block + n * v + 2 * n

    def flops_per_token(self, seq_len: int | None = None) -> float:
        """Training FLOPs per token: 6 x matmul params + causal attention (fwd 2*S*n per layer x 3)."""
        s = seq_len or self.block_size
        n = self.n_embd
        matmul = self.n_layer * 12 * n * n + n * self.vocab_size
        attn = self.n_layer * 2 * s * n  # QK^T and PV with the causal half counted
        return 6.0 * matmul + 6.0 * attn


def _seed_for(config: GPTConfig, layer: int, role: int) -> int:
    # Per-(layer, role) seed; same derivation as the reference (gpt.py:76-77)
    # so equal seeds give equal weights in both frameworks.
    return (config.seed * 1_000_003 + layer * 97 + role) % (2**31 - 1)


class CausalSelfAttention(nn.Module):
    """Heads sharded over the TP group: QKV column-parallel, output projection row-parallel."""

    def __init__(self, config: GPTConfig, layer: int, tp_group=None, device=None, dtype=None):
        super().__init__()
        tp = comm.get_world_size(tp_group)
        if config.n_head % tp:
            raise ValueError(f"n_head={config.n_head} not divisible by tp_size={tp}")
        self.n_head_local = config.n_head // tp
        self.head_dim = config.head_dim
        self.qkv = ColumnParallelLinear(config.n_embd, 3 * config.n_embd, bias=config.bias, group=tp_group,
                                        seed=_seed_for(config, layer, 0), device=device, dtype=dtype)
        self.proj = RowParallelLinear(config.n_embd, config.n_embd, bias=config.bias, input_is_parallel=True,
                                      group=tp_group, seed=_seed_for(config, layer, 1), device=device, dtype=dtype)

    def forward(self, x):
        B, S, _ = x.shape
        q, k, v = self.qkv(x).view(B, S, self.n_head_local, 3, self.head_dim).unbind(dim=3)
        y = F.scaled_dot_product_attention(q.transpose(1, 2), k.transpose(1, 2), v.transpose(1, 2), is_causal=True)
        return self.proj(y.transpose(1, 2).reshape(B, S, self.n_head_local * self.head_dim))


class MLP(nn.Module):
    def __init__(self, config: GPTConfig, layer: int, tp_group=None, device=None, dtype=None):
        super().__init__()
        self.fc = ColumnParallelLinear(config.n_embd, 4 * config.n_embd, bias=config.bias, group=tp_group,
                                       seed=_seed_for(config, layer, 2), device=device, dtype=dtype)
        self.proj = RowParallelLinear(4 * config.n_embd, config.n_embd, bias=config.bias, input_is_parallel=True,
                                      group=tp_group, seed=_seed_for(config, layer, 3), device=device, dtype=dtype)

    def forward(self, x):
        return self.proj(F.gelu(self.fc(x), approximate="tanh"))


class Block(nn.Module):
    """Pre-norm transformer block; also the default FSDP unit."""

    def __init__(self, config: GPTConfig, layer: int, tp_group=None, device=None, dtype=None):
        super().__init__()
        self.layer = layer
        self.tp_group = tp_group
        self.ln1 = nn.LayerNorm(config.n_embd, device=device, dtype=dtype)
        self.attn = CausalSelfAttention(config, layer, tp_group, device, dtype)
        self.ln2 = nn.LayerNorm(config.n_embd, device=device, dtype=dtype)
        self.mlp = MLP(config, layer, tp_group, device, dtype)

    def forward(self, x):
        from . import fused_gpt

        if fused_gpt.should_fuse(x):
            return fused_gpt.block_forward(self, x)
        x = x + self.attn(self.ln1(x))
        return x + self.mlp(self.ln2(x))


class Embedding(nn.Module):
    """Token + learned position embedding (the first pipeline stage)."""

    def __init__(self, config: GPTConfig, tp_group=None, device=None, dtype=None):
        super().__init__()
        self.tp_group = tp_group
        self.wte = VocabParallelEmbedding(config.vocab_size, config.n_embd, group=tp_group,
                                          seed=_seed_for(config, -1, 0), device=device, dtype=dtype)
        gen = torch.Generator(device="cpu").manual_seed(_seed_for(config, -1, 1))
        pos = torch.empty(config.block_size, config.n_embd).normal_(0.0, 0.02, generator=gen)
        self.wpe = nn.Parameter(pos.to(device=device, dtype=dtype))

    def forward(self, input_ids):
        from . import fused_gpt

        if fused_gpt.should_fuse(input_ids):
            return fused_gpt.embedding_forward(self, input_ids)
        return self.wte(input_ids) + self.wpe[: input_ids.size(1)]


class LMHead(nn.Module):
    """Final LayerNorm + column-parallel projection; logits stay vocabulary-sharded.

    ``loss_only=True`` is for the last pipeline stage: ``forward`` then passes the
    hidden states through unchanged and the stage's loss function calls
    :meth:`loss`, which runs LayerNorm, the head GEMM and the vocab-parallel
    cross-entropy as one fused op on the B200 path (the ``[tokens, vocab]``
    logits are never handed between modules).  Parameter names do not change.
    """

    def __init__(self, config: GPTConfig, tp_group=None, device=None, dtype=None):
        super().__init__()
        self.tp_group = tp_group
        self.vocab_size = config.vocab_size
        self.loss_only = False
        self.ln_f = nn.LayerNorm(config.n_embd, device=device, dtype=dtype)
        self.head = ColumnParallelLinear(config.n_embd, config.vocab_size, bias=False, gather_output=False,
                                         group=tp_group, seed=_seed_for(config, -1, 2), device=device, dtype=dtype)

    def forward(self, x):
        if self.loss_only:
            return x
        return self.logits(x)

    def logits(self, x):
        from . import fused_gpt

        if fused_gpt.should_fuse(x):
            return fused_gpt.head_logits(self, x)
        return self.head(self.ln_f(x))

    @property
    def vocab_start(self) -> int:
        tp = comm.get_world_size(self.tp_group)
        return comm.get_rank(self.tp_group) * (self.vocab_size // tp)

    def loss(self, x, targets):
        """LayerNorm + head + vocab-parallel cross-entropy, fused on the B200 path."""
        from . import fused_gpt

        if fused_gpt.should_fuse(x):
            return fused_gpt.head_loss(self, x, targets)
        return vocab_parallel_cross_entropy(self.logits(x), targets, group=self.tp_group,
                                            vocab_start=self.vocab_start)


class GPT(nn.Module):
    """The whole model; ``tp_group=None`` (or size 1) gives the single-device model."""

    def __init__(self, config: GPTConfig, tp_group=None, device=None, dtype=None):
        super().__init__()
        self.config = config
        self.tp_group = tp_group
        self.embedding = Embedding(config, tp_group, device, dtype)
        self.blocks = nn.ModuleList([Block(config, i, tp_group, device, dtype) for i in range(config.n_layer)])
        self.lm_head = LMHead(config, tp_group, device, dtype)

    def forward(self, input_ids, targets=None):
        from . import fused_gpt

        if fused_gpt.should_fuse(input_ids):
            fused_gpt.refresh_shadows(self)
        x = self.embedding(input_ids)
        for block in self.blocks:
            x = block(x)
        if targets is None:
            return self.lm_head.logits(x)
        if fused_gpt.should_fuse(x):
            logits, loss = fused_gpt.head_logits_and_loss(self.lm_head, x, targets)
            return logits, loss
        logits = self.lm_head.logits(x)
        return logits, self.loss(logits, targets)

    def loss(self, logits, targets):
        return vocab_parallel_cross_entropy(logits, targets, group=self.tp_group, vocab_start=self.vocab_start)

    @property
    def vocab_start(self) -> int:
        return self.lm_head.vocab_start

    def num_parameters(self, local: bool = True) -> int:
        n = sum(p.numel() for p in self.parameters())
        return n if local else n * comm.get_world_size(self.tp_group)


def build_pipeline_layers(config: GPTConfig, tp_group=None, device=None, dtype=None) -> list[nn.Module]:
    """``[Embedding, Block x n_layer, LMHead]`` — the sequence a pipeline partitions."""
    layers: list[nn.Module] = [Embedding(config, tp_group, device, dtype)]
    layers += [Block(config, i, tp_group, device, dtype) for i in range(config.n_layer)]
    layers.append(LMHead(config, tp_group, device, dtype))
    return layers


def fused_enabled() -> bool:
    return os.environ.get("MINIDIST_FUSED", "1") not in ("0", "false", "no")
