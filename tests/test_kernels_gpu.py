"""Numerics of the non-GEMM sm_100a kernels against float32 PyTorch references of the same op."""

from __future__ import annotations

import math

import pytest
import torch
import torch.nn.functional as F

from minidist.ops import _native as nat
from minidist.ops import kernels as K

pytestmark = pytest.mark.gpu


def _rel(a, b):
    a, b = a.float(), b.float()
    return ((a - b).abs().max() / b.abs().max().clamp(min=1e-6)).item()


@pytest.mark.parametrize("M,C", [(1000, 768), (100, 256), (300, 1024), (2049, 512), (257, 1600), (64, 2560),
                                 (33, 4096)])
def test_layernorm(M, C):
    torch.manual_seed(0)
    x = (torch.randn(M, C, device="cuda") * 2 + 0.5).bfloat16()
    g = torch.randn(C, device="cuda") * 0.5 + 1
    b = torch.randn(C, device="cuda") * 0.1
    y, mu, rs = K.layernorm_fwd(x, g, b)
    xf = x.float().requires_grad_(True)
    gf, bf = g.clone().requires_grad_(True), b.clone().requires_grad_(True)
    ref = F.layer_norm(xf, (C,), gf, bf, 1e-5)
    nat.check_status()
    assert _rel(y, ref) < 1e-2
    dy = torch.randn(M, C, device="cuda").bfloat16()
    rg = torch.randn(M, C, device="cuda").bfloat16()
    ref.backward(dy.float())
    dg = torch.zeros(C, device="cuda")
    db = torch.zeros(C, device="cuda")
    cr = torch.zeros(C, device="cuda")
    co = torch.zeros(C, device="cuda")
    dx = K.layernorm_bwd(dy, x, mu, rs, g, resid_grad=rg, dgamma=dg, dbeta=db, colsum_resid=cr, colsum_out=co)
    torch.cuda.synchronize()
    assert _rel(dx, xf.grad + rg.float()) < 2e-2
    assert _rel(dg, gf.grad) < 1e-3
    assert _rel(db, bf.grad) < 1e-3
    assert _rel(cr, rg.float().sum(0)) < 1e-4
    assert _rel(co, dx.float().sum(0)) < 1e-3
    # accumulate mode doubles
    K.layernorm_bwd(dy, x, mu, rs, g, dgamma=dg, acc_gamma=True)
    assert _rel(dg, 2 * gf.grad) < 1e-3


def _attn_ref(qkv, B, S, H, D):
    q, k, v = qkv.float().view(B, S, H, 3, D).unbind(3)
    q, k, v = (t.transpose(1, 2) for t in (q, k, v))
    y = F.scaled_dot_product_attention(q, k, v, is_causal=True)
    return y.transpose(1, 2).reshape(B * S, H * D)


@pytest.mark.parametrize("impl", ["tc", "mma"])
@pytest.mark.parametrize("B,S,H,D", [(2, 256, 3, 64), (1, 200, 2, 64), (1, 192, 2, 80), (2, 128, 2, 128),
                                     (1, 1024, 4, 64), (2, 333, 2, 128), (2, 333, 3, 80), (2, 160, 4, 32)])
def test_attention(B, S, H, D, impl):
    torch.manual_seed(1)
    qkv = torch.randn(B * S, 3 * H * D, device="cuda").bfloat16()
    y, lse = K.attention_fwd(qkv, B, S, H, D, impl=impl)
    qf = qkv.float().requires_grad_(True)
    ref = _attn_ref(qf, B, S, H, D)
    nat.check_status()
    assert _rel(y, ref) < 2e-2
    # lse check against an explicit computation
    q, k, _ = qf.detach().view(B, S, H, 3, D).unbind(3)
    s = torch.einsum("bqhd,bkhd->bhqk", q, k) / math.sqrt(D)
    s = s.masked_fill(torch.triu(torch.ones(S, S, dtype=torch.bool, device="cuda"), 1), float("-inf"))
    assert _rel(lse, torch.logsumexp(s, -1)) < 1e-3
    dy = torch.randn(B * S, H * D, device="cuda").bfloat16()
    ref.backward(dy.float())
    dqkv = K.attention_bwd(qkv, y, dy, lse, B, S, H, D, impl=impl)
    nat.check_status()
    assert _rel(dqkv, qf.grad) < 3e-2


def test_attention_fwd_tc_many_tiles():
    """Persistent tcgen05 forward with several work items per CTA, padded row stride, large logits."""
    torch.manual_seed(3)
    B, S, H, D = 4, 1024, 12, 64  # 384 work items over 148 CTAs
    buf = torch.randn(B * S, 3 * H * D + 64, device="cuda").bfloat16() * 3
    qkv = buf[:, : 3 * H * D]
    y, lse = K.attention_fwd(qkv, B, S, H, D, impl="tc")
    y2, lse2 = K.attention_fwd(qkv, B, S, H, D, impl="mma")
    nat.check_status()
    ref = _attn_ref(qkv, B, S, H, D)
    assert _rel(y, ref) < 2e-2
    assert _rel(y, y2) < 2e-2
    assert _rel(lse, lse2) < 1e-3
    dy = torch.randn(B * S, H * D, device="cuda").bfloat16()
    g1 = K.attention_bwd(qkv, y, dy, lse, B, S, H, D, impl="tc")
    g2 = K.attention_bwd(qkv, y, dy, lse, B, S, H, D, impl="mma")
    nat.check_status()
    assert _rel(g1, g2) < 2e-2


@pytest.mark.parametrize("D", [64, 80, 128])
def test_attention_fwd_tc_output_tiles(D):
    """The tcgen05 forward stores each output tile with a bulk tensor store from shared memory:
    rows past S (here S = 1000, B = 2: the next sequence's rows follow) and, at d = 80, columns
    past the head (the next head follows) must be clipped, and the row padding of a strided
    output must stay untouched.  Several work items per CTA exercise the Q/O buffer reuse."""
    torch.manual_seed(5)
    B, S, H = 2, 1000, 12
    qkv = (torch.randn(B * S, 3 * H * D, device="cuda") * 2).bfloat16()
    buf = torch.full((B * S, H * D + 64), 7.0, device="cuda").bfloat16()
    out = buf[:, : H * D]
    lse = torch.empty(B, H, S, device="cuda")
    rc = nat.lib().md_attn_fwd_tc(qkv.data_ptr(), qkv.stride(0), out.data_ptr(), out.stride(0), lse.data_ptr(), B, H,
                                  S, D, 1.0 / math.sqrt(D), nat.status_ptr(qkv.device), nat.stream_ptr())
    nat.check(rc, "md_attn_fwd_tc")
    torch.cuda.synchronize()
    nat.check_status()
    assert bool((buf[:, H * D:] == 7.0).all())
    ref = _attn_ref(qkv, B, S, H, D)
    assert _rel(out, ref) < 2e-2
    q, k, _ = qkv.float().view(B, S, H, 3, D).unbind(3)
    s = torch.einsum("bqhd,bkhd->bhqk", q, k) / math.sqrt(D)
    s = s.masked_fill(torch.triu(torch.ones(S, S, dtype=torch.bool, device="cuda"), 1), float("-inf"))
    assert _rel(lse, torch.logsumexp(s, -1)) < 1e-3


@pytest.mark.parametrize("D", [80, 128])
def test_attention_bwd_tc_wide_heads_many_tiles(D):
    """The head_dim 80 / 128 tcgen05 backward (64-query blocks, dQ^T in TMEM) with several work
    items per CTA and a padded row stride, against the mma.sync backward and fp32 autograd."""
    torch.manual_seed(4)
    B, S, H = 2, 1280, 16  # 10 key tiles x 32 heads = 320 items over 148 CTAs
    buf = torch.randn(B * S, 3 * H * D + 64, device="cuda").bfloat16()
    qkv = buf[:, : 3 * H * D]
    y, lse = K.attention_fwd(qkv, B, S, H, D, impl="tc")
    dy = torch.randn(B * S, H * D, device="cuda").bfloat16()
    g1 = K.attention_bwd(qkv, y, dy, lse, B, S, H, D, impl="tc")
    g2 = K.attention_bwd(qkv, y, dy, lse, B, S, H, D, impl="mma")
    nat.check_status()
    assert _rel(g1, g2) < 2e-2
    qf = qkv.float().requires_grad_(True)
    _attn_ref(qf, B, S, H, D).backward(dy.float())
    assert _rel(g1, qf.grad) < 3e-2


def test_embedding_and_colsum():
    torch.manual_seed(2)
    V, C, B, S = 1000, 768, 4, 64
    wte = torch.randn(V, C, device="cuda").bfloat16()
    wpe = torch.randn(S + 16, C, device="cuda").bfloat16()
    ids = torch.randint(0, V, (B, S), device="cuda")
    out = K.embedding_fwd(ids, wte, wpe[:S], S)
    ref = wte.float()[ids].reshape(B * S, C) + wpe.float()[:S].repeat(B, 1)
    assert _rel(out, ref) < 1e-2
    dx = torch.randn(B * S, C, device="cuda").bfloat16()
    dwte = torch.zeros(V, C, device="cuda")
    K.embedding_bwd_wte(ids, dx, dwte)
    ref_w = torch.zeros(V, C, device="cuda").index_add_(0, ids.reshape(-1), dx.float())
    assert _rel(dwte, ref_w) < 1e-5
    dwpe = torch.zeros(S, C, device="cuda")
    K.embedding_bwd_wpe(dx, dwpe, B, S, accumulate=False)
    assert _rel(dwpe, dx.float().view(B, S, C).sum(0)) < 1e-5
    cs = torch.zeros(C, device="cuda")
    K.colsum(dx, cs)
    nat.check_status()
    assert _rel(cs, dx.float().sum(0)) < 1e-5


def test_fused_adamw_matches_torch():
    from minidist.optim import FusedAdamW

    torch.manual_seed(3)
    ps = [torch.randn(n, device="cuda", requires_grad=True) for n in (1000, 65537, 7, 4096 * 3)]
    qs = [p.detach().clone().requires_grad_(True) for p in ps]
    a = FusedAdamW(ps, lr=1e-3, weight_decay=0.1)
    b = torch.optim.AdamW(qs, lr=1e-3, weight_decay=0.1)
    for _ in range(3):
        for p, q in zip(ps, qs):
            g = torch.randn_like(p)
            p.grad, q.grad = g.clone(), g.clone()
        a.step()
        b.step()
    for p, q in zip(ps, qs):
        assert _rel(p, q) < 1e-5


@pytest.mark.parametrize("M,V,col_offset", [(300, 1003, 0), (64, 50257, 0), (129, 517, 1000)])
def test_ce_backward_matches_fp32(M, V, col_offset):
    """(softmax - onehot) * g * scale from stored bf16 logits, incl. a ragged vocabulary and a vocab shard."""
    from minidist.ops import gemm as G

    torch.manual_seed(7)
    logits = G.empty_padded(M, V, device="cuda")
    logits.copy_(torch.randn(M, V, device="cuda") * 3)
    lf = logits.float()
    lse = torch.logsumexp(lf, dim=1)
    # Targets inside and outside this shard's columns [col_offset, col_offset + V).
    target = torch.randint(0, V, (M,), device="cuda") + col_offset
    target[::5] = col_offset + V + 3 if col_offset else target[::5]
    g = torch.tensor([0.75], device="cuda")
    out = K.ce_backward(logits, lse, target, g, 1.0 / M, V, col_offset=col_offset)
    nat.check_status()
    want = torch.softmax(lf, dim=1)
    local = target - col_offset
    inside = (local >= 0) & (local < V)
    want[inside.nonzero().squeeze(1), local[inside]] -= 1.0
    want *= 0.75 / M
    assert _rel(out, want) < 1e-2
