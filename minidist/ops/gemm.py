"""Python front end of the tcgen05 GEMM (csrc/gemm_sm100.cu).

The three products of a linear layer map onto one kernel with different
operand majors, so no operand is ever transposed in memory:

=========  ====================  =========  =========
product    shape                 A          B
=========  ====================  =========  =========
forward    y[M,N]  = x W^T       x K-major  W K-major
dgrad      dx[M,K] = dy W        dy K-major W MN-major
wgrad      dW[N,K] = dy^T x      dy MN-major x MN-major
=========  ====================  =========  =========
"""

from __future__ import annotations

import ctypes
import os

import torch

from . import _native as nat

EPI_BF16, EPI_F32, EPI_DGELU, EPI_CE = 0, 1, 2, 3
TILE_M, TILE_N = 128, 256
CE_SLAB = 128  # the kEpiCE epilogue keeps statistics per 128-column slab

# Optional overrides of the kernel's own tile choices (0 = let the kernel choose).
_ENV_CG = int(os.environ.get("MINIDIST_GEMM_CTA_GROUP", "0"))
_ENV_EW = int(os.environ.get("MINIDIST_GEMM_EPI_WARPS", "0"))
# Split-K weight gradients: fixed-order workspace reduction when set, fp32
# atomic accumulation into the gradient otherwise (faster; none of the
# split-K outputs is a replicated tensor-parallel parameter).
_DETERMINISTIC = os.environ.get("MINIDIST_DETERMINISTIC", "0") not in ("0", "", "false", "no")


def _vp(t):
    return None if t is None else ctypes.c_void_p(t.data_ptr())


def gemm(
    A: torch.Tensor,
    B: torch.Tensor,
    D: torch.Tensor,
    *,
    M: int,
    N: int,
    K: int,
    lda: int,
    ldb: int,
    ldd: int,
    a_mn: bool = False,
    b_mn: bool = False,
    epi: int = EPI_BF16,
    alpha: float = 1.0,
    beta: bool = False,
    gelu: bool = False,
    bias: torch.Tensor | None = None,
    aux: torch.Tensor | None = None,
    ldaux: int = 0,
    resid: torch.Tensor | None = None,
    ldres: int = 0,
    k_splits: int = 1,
    ce: tuple | None = None,
    ce_col_offset: int = 0,
    num_sms: int = 0,
    cta_group: int = 0,
    epi_warps: int = 0,
    colsum: torch.Tensor | None = None,
    dot: tuple | None = None,
    stream: torch.cuda.Stream | None = None,
) -> None:
    """Raw launcher; see ``struct MdGemmParams`` for the meaning of each field."""
    p = nat.GemmParams()
    p.A, p.B, p.D = A.data_ptr(), B.data_ptr(), D.data_ptr()
    p.lda, p.ldb, p.ldd = lda, ldb, ldd
    p.M, p.N, p.K = M, N, K
    p.a_mn_major, p.b_mn_major = int(a_mn), int(b_mn)
    p.epi = epi
    p.alpha = alpha
    p.beta = int(beta)
    p.gelu = int(gelu)
    p.bias = None if bias is None else bias.data_ptr()
    p.aux = None if aux is None else aux.data_ptr()
    p.ldaux = ldaux
    p.resid = None if resid is None else resid.data_ptr()
    p.ldres = ldres
    ws = None
    if epi == EPI_F32 and k_splits > 1 and _DETERMINISTIC:
        ldws = (N + 3) // 4 * 4
        ws = torch.empty(k_splits * M * ldws, dtype=torch.float32, device=D.device)
        p.workspace = ws.data_ptr()
        p.ldws = ldws
    p.k_splits = k_splits
    if ce is not None:
        target, cmax, csum, ctgt = ce
        p.ce_target, p.ce_max, p.ce_sum, p.ce_tgt = (
            target.data_ptr(), cmax.data_ptr(), csum.data_ptr(), ctgt.data_ptr())
    p.ce_col_offset = ce_col_offset
    p.num_sms = num_sms
    p.cta_group = cta_group or _ENV_CG
    p.epi_warps = epi_warps or _ENV_EW
    p.colsum = None if colsum is None else colsum.data_ptr()
    if dot is not None:
        dot_in, dot_out, group, seq = dot
        p.dot_in, p.lddot, p.dot_out, p.dot_group, p.dot_seq = (
            dot_in.data_ptr(), _ld(dot_in), dot_out.data_ptr(), group, seq)
    p.status = nat.status_ptr(D.device)
    rc = nat.lib().md_gemm(ctypes.byref(p), ctypes.c_void_p(nat.stream_ptr(stream)))
    nat.check(rc, f"md_gemm(M={M},N={N},K={K},a_mn={a_mn},b_mn={b_mn},epi={epi})")
    if ws is not None:
        # Keep the workspace alive until the reduce kernel has consumed it.
        ws.record_stream(stream if stream is not None else torch.cuda.current_stream())


def empty_padded(rows: int, cols: int, dtype=torch.bfloat16, device=None) -> torch.Tensor:
    """``[rows, cols]`` view of a buffer whose row stride is a multiple of 16 bytes."""
    mult = 16 // torch.empty((), dtype=dtype).element_size()
    ld = (cols + mult - 1) // mult * mult
    buf = torch.empty(rows, ld, dtype=dtype, device=device)
    return buf if ld == cols else buf[:, :cols]


def _ld(t: torch.Tensor) -> int:
    assert t.dim() == 2 and t.stride(1) == 1, "expected a row-major 2-D tensor"
    return t.stride(0)


def pick_k_splits(units: int, k_blocks: int, sms: int) -> int:
    """Split-K factor that best fills ``sms`` SMs (each split keeps >= 8 k-blocks)."""
    if units >= sms:
        return 1
    best, best_eff = 1, 0.0
    for s in range(1, 17):
        if s > 1 and k_blocks // s < 8:
            break
        work = units * s
        waves = -(-work // sms)
        eff = work / (waves * sms) - 0.01 * s
        if eff > best_eff + 1e-9:
            best, best_eff = s, eff
    return best


def linear_fwd(
    x: torch.Tensor,
    w: torch.Tensor,
    bias: torch.Tensor | None = None,
    *,
    gelu: bool = False,
    resid: torch.Tensor | None = None,
    out: torch.Tensor | None = None,
    preact_out: torch.Tensor | None = None,
) -> torch.Tensor | tuple[torch.Tensor, torch.Tensor]:
    """``y = [resid +] act(x @ w^T + bias)`` in bf16.  With ``gelu`` also returns the pre-activation."""
    M, K = x.shape
    N = w.shape[0]
    if out is None:
        out = empty_padded(M, N, device=x.device)
    pre = None
    if gelu:
        pre = preact_out if preact_out is not None else empty_padded(M, N, device=x.device)
    gemm(x, w, out, M=M, N=N, K=K, lda=_ld(x), ldb=_ld(w), ldd=_ld(out), epi=EPI_BF16,
         bias=bias, gelu=gelu, aux=pre, ldaux=_ld(pre) if pre is not None else 0,
         resid=resid, ldres=_ld(resid) if resid is not None else 0)
    return (out, pre) if gelu else out


def linear_dgrad(
    dy: torch.Tensor,
    w: torch.Tensor,
    *,
    gelu_preact: torch.Tensor | None = None,
    out: torch.Tensor | None = None,
    colsum_partial: torch.Tensor | None = None,
    dot: tuple | None = None,
) -> torch.Tensor:
    """``dx = dy @ w`` (bf16); with ``gelu_preact`` returns ``(dy @ w) * gelu'(preact)``.

    ``colsum_partial`` (with ``gelu_preact``): fp32 ``[ceil(M/32) * K]`` that receives the
    per-32-row column sums of the result (finish with ``kernels.colsum_final``).
    ``dot = (o, out, group, seq)`` (without ``gelu_preact``): also writes the row-wise dot products
    of the result with ``o`` over each ``group`` columns (32 / 64 / 128) to
    ``out[((row // seq) * (K // group) + g) * seq + row % seq]`` (fp32) -- the attention
    backward's ``delta`` when the result is dO and ``o`` the attention output."""
    M, N = dy.shape
    K = w.shape[1]
    if out is None:
        out = empty_padded(M, K, device=dy.device)
    epi = EPI_DGELU if gelu_preact is not None else EPI_BF16
    if colsum_partial is not None and (epi != EPI_DGELU or colsum_partial.numel() < -(-M // 32) * K):
        raise ValueError("colsum_partial needs gelu_preact and ceil(M/32) * K elements")
    gemm(dy, w, out, M=M, N=K, K=N, lda=_ld(dy), ldb=_ld(w), ldd=_ld(out), b_mn=True, epi=epi,
         aux=gelu_preact, ldaux=_ld(gelu_preact) if gelu_preact is not None else 0, colsum=colsum_partial,
         dot=dot)
    return out


def linear_wgrad(
    dy: torch.Tensor,
    x: torch.Tensor,
    out: torch.Tensor,
    *,
    accumulate: bool = False,
    k_splits: int | None = None,
) -> torch.Tensor:
    """``out[N,K] (+)= dy^T @ x`` in fp32 (dy [M,N], x [M,K], both bf16)."""
    M, N = dy.shape
    K = x.shape[1]
    if k_splits is None:
        units = -(-N // (2 * TILE_M if N >= 2304 else TILE_M)) * -(-K // TILE_N)
        k_splits = pick_k_splits(units, -(-M // 64), nat.num_sms(dy.device))
    gemm(dy, x, out, M=N, N=K, K=M, lda=_ld(dy), ldb=_ld(x), ldd=_ld(out), a_mn=True, b_mn=True,
         epi=EPI_F32, beta=accumulate, k_splits=k_splits)
    return out
