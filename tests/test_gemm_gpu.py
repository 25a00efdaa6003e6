"""tcgen05 GEMM numerics against a float32 PyTorch reference of the same product."""

from __future__ import annotations

import pytest
import torch

from minidist.ops import _native as nat
from minidist.ops import gemm as G

pytestmark = pytest.mark.gpu

SHAPES = [(128, 256, 64), (256, 512, 128), (300, 200, 100), (1024, 768, 768), (4096, 2304, 768), (130, 50257 // 64, 96)]


def _rel(a: torch.Tensor, b: torch.Tensor) -> float:
    a, b = a.float(), b.float()
    return ((a - b).abs().max() / b.abs().max().clamp(min=1e-6)).item()


def _bf16(rows, cols, scale=1.0):
    """Random bf16 matrix whose row stride is padded to a multiple of 8 elements
    (16 bytes, what TMA needs); ragged logical widths exercise the zero fill."""
    ld = (cols + 7) // 8 * 8
    full = (torch.randn(rows, ld, device="cuda") * scale).to(torch.bfloat16)
    return full[:, :cols]


@pytest.mark.parametrize("M,N,K", SHAPES)
def test_forward_plain(M, N, K):
    torch.manual_seed(0)
    x, w = _bf16(M, K), _bf16(N, K, scale=0.05)
    y = G.linear_fwd(x, w)
    ref = x.float() @ w.float().t()
    nat.check_status()
    assert _rel(y, ref) < 1e-2


@pytest.mark.parametrize("M,N,K", [(256, 512, 128), (1000, 768, 320)])
def test_forward_bias_gelu_residual(M, N, K):
    torch.manual_seed(1)
    x, w = _bf16(M, K), _bf16(N, K, scale=0.05)
    b = torch.randn(N, device="cuda") * 0.1
    y, pre = G.linear_fwd(x, w, b, gelu=True)
    ref_pre = x.float() @ w.float().t() + b
    nat.check_status()
    assert _rel(pre, ref_pre) < 1e-2
    ref = torch.nn.functional.gelu(pre.float(), approximate="tanh")
    assert _rel(y, ref) < 1e-2
    r = _bf16(M, N)
    y2 = G.linear_fwd(x, w, b, resid=r)
    assert _rel(y2, ref_pre + r.float()) < 1e-2


@pytest.mark.parametrize("M,N,K", SHAPES[:5])
def test_dgrad(M, N, K):
    torch.manual_seed(2)
    dy, w = _bf16(M, N), _bf16(N, K, scale=0.05)
    dx = G.linear_dgrad(dy, w)
    nat.check_status()
    assert _rel(dx, dy.float() @ w.float()) < 1e-2


def test_dgrad_gelu():
    torch.manual_seed(3)
    M, N, K = 512, 256, 768
    dy, w = _bf16(M, N), _bf16(N, K, scale=0.05)
    h = _bf16(M, K)
    dx = G.linear_dgrad(dy, w, gelu_preact=h)
    hf = h.float().requires_grad_(True)
    torch.nn.functional.gelu(hf, approximate="tanh").backward(dy.float() @ w.float())
    nat.check_status()
    assert _rel(dx, hf.grad) < 2e-2


@pytest.mark.parametrize("M,N,K", SHAPES[:5])
@pytest.mark.parametrize("splits", [1, 3])
def test_wgrad(M, N, K, splits):
    torch.manual_seed(4)
    dy, x = _bf16(M, N), _bf16(M, K)
    out = torch.zeros(N, (K + 3) // 4 * 4, device="cuda")[:, :K]
    G.linear_wgrad(dy, x, out, k_splits=splits)
    ref = dy.float().t() @ x.float()
    nat.check_status()
    assert _rel(out, ref) < 1e-4
    G.linear_wgrad(dy, x, out, accumulate=True, k_splits=splits)
    assert _rel(out, 2 * ref) < 1e-4


def test_wgrad_auto_split_large_reduction():
    torch.manual_seed(5)
    M, N, K = 16384, 768, 768
    dy, x = _bf16(M, N), _bf16(M, K)
    out = torch.empty(N, K, device="cuda")
    G.linear_wgrad(dy, x, out)
    nat.check_status()
    assert _rel(out, dy.float().t() @ x.float()) < 1e-4


@pytest.mark.parametrize("cg", [1, 2])
@pytest.mark.parametrize("a_mn,b_mn", [(False, False), (False, True), (True, True)])
def test_cta_group_variants(cg, a_mn, b_mn):
    """Both tile configurations (1-CTA 128x256, 2-CTA 256x256) for every operand layout, ragged sizes."""
    torch.manual_seed(6)
    M, N, K = 1000, 700, 520
    A = _bf16(K, M) if a_mn else _bf16(M, K)
    B = _bf16(K, N) if b_mn else _bf16(N, K)
    D = torch.zeros(M, (N + 3) // 4 * 4, device="cuda")[:, :N]
    G.gemm(A, B, D, M=M, N=N, K=K, lda=A.stride(0), ldb=B.stride(0), ldd=D.stride(0), a_mn=a_mn, b_mn=b_mn,
           epi=G.EPI_F32, cta_group=cg)
    Af = A.float().t() if a_mn else A.float()
    Bf = B.float() if b_mn else B.float().t()
    nat.check_status()
    assert _rel(D, Af @ Bf) < 1e-4


@pytest.mark.parametrize("M,N,K", [(1000, 384, 640), (4096, 768, 3072), (333, 256, 200)])
def test_dgrad_gelu_fused_bias_colsum(M, N, K):
    """kEpiDGELU's per-32-row column sums + colsum_final equal the column sum of the output."""
    from minidist.ops import kernels as Kn

    dy = torch.randn(M, N, device="cuda").bfloat16()
    w = (torch.randn(N, K, device="cuda") * 0.05).bfloat16()
    h = torch.randn(M, K, device="cuda").bfloat16()
    chunks = -(-M // 32)
    part = torch.full((chunks * K,), float("nan"), device="cuda")
    dx = G.linear_dgrad(dy, w, gelu_preact=h, colsum_partial=part)
    out = torch.full((K,), 0.5, device="cuda")
    Kn.colsum_final(part, chunks, out, accumulate=True)
    want = dx.float().sum(0) + 0.5
    torch.testing.assert_close(out, want, rtol=1e-4, atol=1e-3)
    # The same output as without the fused sums.
    torch.testing.assert_close(dx, G.linear_dgrad(dy, w, gelu_preact=h), rtol=0, atol=0)


@pytest.mark.parametrize("M,N,K,group,seq", [(2048, 768, 768, 64, 1024), (512, 384, 256, 128, 128),
                                             (1024, 256, 96, 32, 256)])
def test_dgrad_fused_rowwise_dot(M, N, K, group, seq):
    """The dot epilogue: delta[(b*G + g)*S + q] = sum over group g of bf16(dy @ w)[row] * o[row]."""
    dy = torch.randn(M, N, device="cuda").bfloat16()
    w = (torch.randn(N, K, device="cuda") * 0.05).bfloat16()
    o = torch.randn(M, K, device="cuda").bfloat16()
    delta = torch.full((M * (K // group),), float("nan"), device="cuda")
    dx = G.linear_dgrad(dy, w, dot=(o, delta, group, seq))
    nat.check_status()
    prod = (dx.float() * o.float()).reshape(M // seq, seq, K // group, group).sum(-1)  # [B, S, G]
    want = prod.permute(0, 2, 1).reshape(-1)
    torch.testing.assert_close(delta, want, rtol=1e-4, atol=1e-3)
    torch.testing.assert_close(dx, G.linear_dgrad(dy, w), rtol=0, atol=0)
