"""Thin Python wrappers over the non-GEMM sm_100a kernels.

Each function validates shapes, allocates outputs with PyTorch's caching
allocator and launches on the current stream.  Kernels: LayerNorm
(csrc/layernorm.cu), flash attention (csrc/attention_sm100.cu on the tcgen05
tensor cores for head_dim 64/128, csrc/attention.cu otherwise), embedding and
column sums (csrc/embedding.cu), cross-entropy pieces (csrc/cross_entropy.cu).
"""

from __future__ import annotations

import math
import os

import torch

from . import _native as nat
from .gemm import empty_padded

_SIGS = {
    "md_ln_fwd": "i:plppplppiifp",
    "md_ln_bwd": "i:plplpppplplpiiip",
    "md_ln_bwd_grid": "i:iii",
    "md_ln_reduce": "i:piiippppip",
    "md_attn_fwd": "i:plplpiiiifp",
    "md_attn_fwd_tc": "i:plplpiiiifpp",
    "md_attn_bwd_tc": "i:plplplppppliiiifpp",
    "md_attn_bwd": "i:plplplppppliiiifp",
    "md_embed_fwd": "i:pplplpliiillip",
    "md_embed_bwd_wte": "i:pplpliillp",
    "md_embed_bwd_wpe": "i:plpliiiip",
    "md_colsum_chunks": "i:ii",
    "md_colsum": "i:pliippip",
    "md_colsum_final": "i:piipip",
    "md_ce_stats": "i:ppiipppppp",
    "md_ce_backward": "i:plpplpfpliip",
    "md_adamw": "i:ppifffffffppipp",
    "md_adamw_chunk": "i:",
    "md_nonfinite": "i:ppipp",
    "md_adamw_entry_bytes": "i:",
    "md_attn_trace_enable": "i:i",
    "md_attn_trace_read": "i:p",
}
for _n, _s in _SIGS.items():
    nat.declare(_n, _s)


def _ld(t: torch.Tensor) -> int:
    assert t.stride(-1) == 1
    return t.stride(0) if t.dim() == 2 else t.stride(-2)


def _s() -> int:
    return nat.stream_ptr()


def _p(t):
    return None if t is None else t.data_ptr()


# ---------------------------------------------------------------------------
# LayerNorm
# ---------------------------------------------------------------------------


def layernorm_fwd(x: torch.Tensor, gamma: torch.Tensor, beta: torch.Tensor, eps: float = 1e-5):
    """``x [M, C]`` bf16 -> ``(y bf16, mean fp32 [M], rstd fp32 [M])``."""
    M, C = x.shape
    y = empty_padded(M, C, device=x.device)
    mean = torch.empty(M, dtype=torch.float32, device=x.device)
    rstd = torch.empty_like(mean)
    rc = nat.lib().md_ln_fwd(x.data_ptr(), _ld(x), gamma.data_ptr(), beta.data_ptr(), y.data_ptr(), _ld(y),
                             mean.data_ptr(), rstd.data_ptr(), M, C, eps, _s())
    nat.check(rc, "md_ln_fwd")
    return y, mean, rstd


def layernorm_bwd(dy, x, mean, rstd, gamma, *, resid_grad=None, dgamma=None, dbeta=None, acc_gamma=False,
                  acc_beta=False, colsum_resid=None, acc_resid=False, colsum_out=None, acc_out=False):
    """LayerNorm backward (+ residual gradient); writes parameter gradients in place.

    Returns ``dx = LN'(dy) + resid_grad``.  ``colsum_resid`` / ``colsum_out``
    (optional fp32 ``[C]``) receive the column sums of ``resid_grad`` and of
    ``dx``; ``acc_*`` selects accumulate vs overwrite for each destination.
    """
    M, C = dy.shape
    dx = empty_padded(M, C, device=dy.device)
    extra = colsum_resid is not None or colsum_out is not None
    nacc = 4 if extra else 2
    lib = nat.lib()
    grid = lib.md_ln_bwd_grid(M, C, nacc)
    partials = torch.empty(grid * nacc * C, dtype=torch.float32, device=dy.device)
    rc = lib.md_ln_bwd(dy.data_ptr(), _ld(dy), x.data_ptr(), _ld(x), mean.data_ptr(), rstd.data_ptr(),
                       gamma.data_ptr(), _p(resid_grad), _ld(resid_grad) if resid_grad is not None else 0,
                       dx.data_ptr(), _ld(dx), partials.data_ptr(), nacc, M, C, _s())
    nat.check(rc, "md_ln_bwd")
    mask = int(acc_gamma) | (int(acc_beta) << 1) | (int(acc_resid) << 2) | (int(acc_out) << 3)
    rc = lib.md_ln_reduce(partials.data_ptr(), grid, nacc, C, _p(dgamma), _p(dbeta), _p(colsum_resid),
                          _p(colsum_out), mask, _s())
    nat.check(rc, "md_ln_reduce")
    return dx


# ---------------------------------------------------------------------------
# Attention
# ---------------------------------------------------------------------------


# MINIDIST_ATTN_FWD=mma / MINIDIST_ATTN_BWD=mma select the warp-level mma.sync
# kernels for every head size (the tests check the two against each other).
_ATTN_FWD = os.environ.get("MINIDIST_ATTN_FWD", "tc")
_ATTN_BWD = os.environ.get("MINIDIST_ATTN_BWD", "tc")


def attention_fwd(qkv: torch.Tensor, B: int, S: int, H: int, D: int, impl: str | None = None):
    """Causal attention on the per-head interleaved ``qkv [B*S, 3*H*D]``; returns ``(out [B*S, H*D], lse)``."""
    out = empty_padded(B * S, H * D, device=qkv.device)
    lse = torch.empty(B, H, S, dtype=torch.float32, device=qkv.device)
    impl = impl or _ATTN_FWD
    if impl == "tc" and D in (64, 80, 128):  # d = 80 runs the d = 128 kernel on zero-padded boxes
        rc = nat.lib().md_attn_fwd_tc(qkv.data_ptr(), _ld(qkv), out.data_ptr(), _ld(out), lse.data_ptr(), B, H, S,
                                      D, 1.0 / math.sqrt(D), nat.status_ptr(qkv.device), _s())
        nat.check(rc, f"md_attn_fwd_tc(D={D})")
    else:
        rc = nat.lib().md_attn_fwd(qkv.data_ptr(), _ld(qkv), out.data_ptr(), _ld(out), lse.data_ptr(), B, H, S, D,
                                   1.0 / math.sqrt(D), _s())
        nat.check(rc, f"md_attn_fwd(D={D})")
    return out, lse


def attention_bwd_impl() -> str:
    """The attention backward in use: ``"tc"`` (tcgen05, d = 64 / 80 / 128) or ``"mma"``."""
    return _ATTN_BWD


def attention_pipeline_trace(fn) -> torch.Tensor:
    """Run ``fn`` (one tcgen05 attention launch) with the kernel's pipeline trace on and return
    CTA 0's ``clock64()`` stamps as int64 [64 key blocks, 32 slots] (0 = not recorded).

    Analysis only: the trace costs a global store per stamp.  Slot meanings are listed beside
    the kernels' MD_FTRACE / MD_TRACE macros."""
    nat.check(nat.lib().md_attn_trace_enable(1), "md_attn_trace_enable")
    try:
        fn()
        torch.cuda.synchronize()
        out = torch.zeros(64, 32, dtype=torch.int64)
        nat.check(nat.lib().md_attn_trace_read(out.data_ptr()), "md_attn_trace_read")
    finally:
        nat.lib().md_attn_trace_enable(0)
    return out


def attention_bwd(qkv, out, dout, lse, B: int, S: int, H: int, D: int, dqkv: torch.Tensor | None = None,
                  impl: str | None = None, delta: torch.Tensor | None = None):
    """Gradients w.r.t. ``qkv`` in the same interleaved layout.

    ``delta``: ``rowsum(dout * out)`` per (batch, head, query), fp32 ``[B*H*S]``, when the caller
    already has it (the dO-producing GEMM's dot epilogue, ``gemm.linear_dgrad(dot=...)``)."""
    if dqkv is None:
        dqkv = empty_padded(B * S, 3 * H * D, device=qkv.device)
    have_delta = delta is not None
    if delta is None:
        delta = torch.empty(B * H * S, dtype=torch.float32, device=qkv.device)
    dqacc = torch.empty(B * S, H * D, dtype=torch.float32, device=qkv.device)
    impl = impl or _ATTN_BWD
    if impl == "tc" and D in (64, 80, 128):  # d = 80 runs the d = 128 kernel on zero-padded boxes
        rc = nat.lib().md_attn_bwd_tc(qkv.data_ptr(), _ld(qkv), None if have_delta else out.data_ptr(), _ld(out),
                                      dout.data_ptr(), _ld(dout),
                                      lse.data_ptr(), delta.data_ptr(), dqacc.data_ptr(), dqkv.data_ptr(), _ld(dqkv),
                                      B, H, S, D, 1.0 / math.sqrt(D), nat.status_ptr(qkv.device), _s())
        nat.check(rc, f"md_attn_bwd_tc(D={D})")
    else:
        rc = nat.lib().md_attn_bwd(qkv.data_ptr(), _ld(qkv), out.data_ptr(), _ld(out), dout.data_ptr(), _ld(dout),
                                   lse.data_ptr(), delta.data_ptr(), dqacc.data_ptr(), dqkv.data_ptr(), _ld(dqkv),
                                   B, H, S, D, 1.0 / math.sqrt(D), _s())
        nat.check(rc, f"md_attn_bwd(D={D})")
    return dqkv


# ---------------------------------------------------------------------------
# Embedding / column sums
# ---------------------------------------------------------------------------


def embedding_fwd(ids: torch.Tensor, wte: torch.Tensor, wpe: torch.Tensor | None, S: int, vocab_start: int = 0):
    """``wte[ids - vocab_start]`` (zero outside the shard) ``+ wpe[position]`` as bf16 ``[tokens, C]``."""
    ids = ids.reshape(-1)
    M = ids.numel()
    C = wte.shape[1]
    out = empty_padded(M, C, device=ids.device)
    rc = nat.lib().md_embed_fwd(ids.data_ptr(), wte.data_ptr(), _ld(wte), _p(wpe),
                                _ld(wpe) if wpe is not None else 0, out.data_ptr(), _ld(out), M, S, C, vocab_start,
                                wte.shape[0], int(wpe is not None), _s())
    nat.check(rc, "md_embed_fwd")
    return out


def embedding_bwd_wte(ids: torch.Tensor, dx: torch.Tensor, dwte: torch.Tensor, vocab_start: int = 0) -> None:
    """``dwte[ids - vocab_start] += dx`` (fp32, atomic)."""
    M, C = dx.shape
    rc = nat.lib().md_embed_bwd_wte(ids.reshape(-1).data_ptr(), dx.data_ptr(), _ld(dx), dwte.data_ptr(), _ld(dwte),
                                    M, C, vocab_start, dwte.shape[0], _s())
    nat.check(rc, "md_embed_bwd_wte")


def embedding_bwd_wpe(dx: torch.Tensor, dwpe: torch.Tensor, B: int, S: int, accumulate: bool) -> None:
    C = dx.shape[1]
    rc = nat.lib().md_embed_bwd_wpe(dx.data_ptr(), _ld(dx), dwpe.data_ptr(), _ld(dwpe), B, S, C, int(accumulate), _s())
    nat.check(rc, "md_embed_bwd_wpe")


def colsum(x: torch.Tensor, out: torch.Tensor, accumulate: bool = False) -> torch.Tensor:
    """``out[n] (+)= sum_m x[m, n]`` (bf16 in, fp32 out, fixed summation order)."""
    M, N = x.shape
    lib = nat.lib()
    partial = torch.empty(lib.md_colsum_chunks(M, N) * N, dtype=torch.float32, device=x.device)
    rc = lib.md_colsum(x.data_ptr(), _ld(x), M, N, partial.data_ptr(), out.data_ptr(), int(accumulate), _s())
    nat.check(rc, "md_colsum")
    return out


def colsum_final(partial: torch.Tensor, chunks: int, out: torch.Tensor, accumulate: bool = False) -> torch.Tensor:
    """``out[n] (+)= sum_c partial[c, n]`` over ``chunks`` fp32 partial rows (fixed order)."""
    N = out.numel()
    rc = nat.lib().md_colsum_final(partial.data_ptr(), chunks, N, out.data_ptr(), int(accumulate), _s())
    nat.check(rc, "md_colsum_final")
    return out


# ---------------------------------------------------------------------------
# Cross-entropy pieces around the kEpiCE LM-head GEMM
# ---------------------------------------------------------------------------


def ce_stats(tmax, tsum, tgt_logit=None, finish: bool = True):
    """Combine column-tile statistics; returns ``(row_max, row_sum, lse, loss)`` (last two if ``finish``)."""
    tiles, M = tmax.shape
    dev = tmax.device
    rmax = torch.empty(M, dtype=torch.float32, device=dev)
    rsum = torch.empty_like(rmax)
    lse = torch.empty_like(rmax) if finish else None
    loss = torch.empty_like(rmax) if finish else None
    rc = nat.lib().md_ce_stats(tmax.data_ptr(), tsum.data_ptr(), tiles, M, rmax.data_ptr(), rsum.data_ptr(),
                               _p(tgt_logit), _p(lse), _p(loss), _s())
    nat.check(rc, "md_ce_stats")
    return rmax, rsum, lse, loss


def ce_backward(logits, lse, target, grad_out, scale: float, V: int, col_offset: int = 0, out=None):
    """``(softmax - onehot) * grad_out * scale`` as bf16, recomputed from the stored logits."""
    M = logits.shape[0]
    if out is None:
        out = empty_padded(M, V, device=logits.device)
    rc = nat.lib().md_ce_backward(logits.data_ptr(), _ld(logits), lse.data_ptr(), target.data_ptr(), col_offset,
                                  _p(grad_out), scale, out.data_ptr(), _ld(out), M, V, _s())
    nat.check(rc, "md_ce_backward")
    return out
