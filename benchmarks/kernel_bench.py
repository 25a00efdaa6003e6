#!/usr/bin/env python3
"""Microbenchmarks of the sm_100a kernels against the library equivalents.

    python benchmarks/kernel_bench.py --op gemm --shape 16384,2304,768
    python benchmarks/kernel_bench.py --op attention --shape 16,12,1024,64
    python benchmarks/kernel_bench.py --op layernorm --shape 16384,768
    python benchmarks/kernel_bench.py --op all

Times are CUDA-event averages after warm-up on the launching stream.  GEMM
rows report forward (y = x W^T), data-gradient (dx = dy W) and weight-gradient
(dW = dy^T x) throughput next to cuBLAS (torch.matmul) for the same product.
Attention rows compare with torch's scaled_dot_product_attention (cuDNN / flash
backends).  ``--op gemm --shape M,N,K --which fwd --iters 3`` is the small case
used for ncu captures of one GEMM launch.
"""

from __future__ import annotations

import argparse
import sys
from pathlib import Path

import torch
import torch.nn.functional as F

sys.path.insert(0, str(Path(__file__).resolve().parent.parent))

from minidist.ops import _native as nat  # noqa: E402
from minidist.ops import gemm as G  # noqa: E402
from minidist.ops import kernels as K  # noqa: E402


def timed(fn, iters: int, warmup: int = 3) -> float:
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    for _ in range(iters):
        fn()
    b.record()
    b.synchronize()
    return a.elapsed_time(b) / 1e3 / iters


def bench_gemm(M, N, K, iters, cta_group=0, which="fwd,dgrad,wgrad"):
    x = torch.randn(M, K, device="cuda").bfloat16()
    w = (torch.randn(N, K, device="cuda") * 0.02).bfloat16()
    dy = G.empty_padded(M, N, device="cuda")  # row strides must be 16-byte multiples (N = 50257)
    dy.copy_(torch.randn(M, N, device="cuda"))
    out = G.empty_padded(M, N, device="cuda")
    dx = torch.empty(M, K, device="cuda", dtype=torch.bfloat16)
    dw = torch.empty(N, K, device="cuda")
    fl = 2.0 * M * N * K
    rows = []
    if "fwd" in which:
        t = timed(lambda: G.gemm(x, w, out, M=M, N=N, K=K, lda=K, ldb=K, ldd=out.stride(0), cta_group=cta_group), iters)
        tc = timed(lambda: torch.matmul(x, w.t()), iters)
        rows.append(("fwd", t, tc))
    if "dgrad" in which:
        t = timed(lambda: G.gemm(dy, w, dx, M=M, N=K, K=N, lda=dy.stride(0), ldb=K, ldd=K, b_mn=True, cta_group=cta_group), iters)
        tc = timed(lambda: torch.matmul(dy, w), iters)
        rows.append(("dgrad", t, tc))
    if "gelu" in which.split(","):
        # fc forward: bias + GELU epilogue storing both the activation and the pre-activation
        bias = torch.randn(N, device="cuda")
        pre = G.empty_padded(M, N, device="cuda")
        t = timed(lambda: G.linear_fwd(x, w, bias, gelu=True, out=out, preact_out=pre), iters)
        bb = bias.bfloat16()
        tc = timed(lambda: F.gelu(torch.addmm(bb, x, w.t()), approximate="tanh"), iters)
        rows.append(("gelu", t, tc))
    if "dgelu" in which.split(","):
        # MLP backward: dgrad with the GELU derivative fused (pre-activation [M, K] read in the epilogue)
        h = torch.randn(M, K, device="cuda").bfloat16()
        t = timed(lambda: G.linear_dgrad(dy, w, gelu_preact=h, out=dx), iters)
        hf = h.float()

        def ref():
            g = torch.matmul(dy, w).float()
            th = torch.tanh(0.7978845608 * (hf + 0.044715 * hf ** 3))
            return g * (0.5 * (1 + th) + 0.5 * hf * (1 - th * th) * 0.7978845608 * (1 + 3 * 0.044715 * hf * hf))
        tc = timed(ref, iters)
        rows.append(("dgelu", t, tc))
    if "wgrad" in which:
        t = timed(lambda: G.linear_wgrad(dy, x, dw), iters)
        tc = timed(lambda: torch.matmul(dy.t(), x), iters)
        rows.append(("wgrad", t, tc))
    nat.check_status()
    for name, t, tc in rows:
        print(f"gemm {name:5s} M={M} N={N} K={K}: {t * 1e6:8.1f} us {fl / t / 1e12:7.1f} TFLOP/s | "
              f"cuBLAS {tc * 1e6:8.1f} us {fl / tc / 1e12:7.1f} TFLOP/s | ratio {tc / t:5.2f}")


def bench_attention(B, H, S, D, iters, fwd_only=False):
    qkv = torch.randn(B * S, 3 * H * D, device="cuda").bfloat16()
    fl_f = 4.0 * B * H * S * S * D / 2
    t = timed(lambda: K.attention_fwd(qkv, B, S, H, D), iters)
    if fwd_only:
        q, k, v = (z.transpose(1, 2).contiguous() for z in qkv.view(B, S, H, 3, D).unbind(3))
        tr = timed(lambda: F.scaled_dot_product_attention(q, k, v, is_causal=True), iters)
        nat.check_status()
        print(f"attention fwd B={B} H={H} S={S} D={D}: {t * 1e6:8.1f} us {fl_f / t / 1e12:6.1f} TFLOP/s | "
              f"torch SDPA {tr * 1e6:8.1f} us {fl_f / tr / 1e12:6.1f} TFLOP/s | ratio {tr / t:5.2f}")
        return
    tm = timed(lambda: K.attention_fwd(qkv, B, S, H, D, impl="mma"), iters)
    y, lse = K.attention_fwd(qkv, B, S, H, D)
    dy = torch.randn_like(y)
    tb = timed(lambda: K.attention_bwd(qkv, y, dy, lse, B, S, H, D), iters)
    tmb = timed(lambda: K.attention_bwd(qkv, y, dy, lse, B, S, H, D, impl="mma"), iters)
    q, k, v = (z.transpose(1, 2) for z in qkv.view(B, S, H, 3, D).unbind(3))
    q, k, v = (z.contiguous().requires_grad_(True) for z in (q, k, v))
    tr = timed(lambda: F.scaled_dot_product_attention(q, k, v, is_causal=True), iters)
    o = F.scaled_dot_product_attention(q, k, v, is_causal=True)
    g = torch.randn_like(o)
    trb = timed(lambda: torch.autograd.grad(o, (q, k, v), g, retain_graph=True), iters)
    nat.check_status()
    print(f"attention fwd B={B} H={H} S={S} D={D}: {t * 1e6:8.1f} us {fl_f / t / 1e12:6.1f} TFLOP/s | "
          f"torch SDPA {tr * 1e6:8.1f} us {fl_f / tr / 1e12:6.1f} TFLOP/s | mma.sync {tm * 1e6:8.1f} us")
    print(f"attention bwd B={B} H={H} S={S} D={D}: {tb * 1e6:8.1f} us {2.5 * fl_f / tb / 1e12:6.1f} TFLOP/s | "
          f"torch SDPA {trb * 1e6:8.1f} us {2.5 * fl_f / trb / 1e12:6.1f} TFLOP/s | mma.sync {tmb * 1e6:8.1f} us")


def bench_layernorm(M, C, iters):
    x = torch.randn(M, C, device="cuda").bfloat16()
    g = torch.ones(C, device="cuda")
    b = torch.zeros(C, device="cuda")
    t = timed(lambda: K.layernorm_fwd(x, g, b), iters)
    y, mu, rs = K.layernorm_fwd(x, g, b)
    dy = torch.randn_like(y)
    dg, db = torch.zeros(C, device="cuda"), torch.zeros(C, device="cuda")
    tb = timed(lambda: K.layernorm_bwd(dy, x, mu, rs, g, resid_grad=dy, dgamma=dg, dbeta=db), iters)
    nat.check_status()
    byt = 2.0 * M * C * 2
    print(f"layernorm fwd M={M} C={C}: {t * 1e6:7.1f} us {byt / t / 1e9:7.0f} GB/s | bwd {tb * 1e6:7.1f} us "
          f"{2 * byt / tb / 1e9:7.0f} GB/s")


def main():
    p = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    p.add_argument("--op", default="all", choices=["all", "gemm", "attention", "layernorm"])
    p.add_argument("--shape", default=None, help="comma-separated problem shape")
    p.add_argument("--iters", type=int, default=20)
    p.add_argument("--cta-group", type=int, default=0)
    p.add_argument("--which", default="fwd,dgrad,wgrad")
    p.add_argument("--fwd-only", action="store_true", help="attention: forward against SDPA only")
    a = p.parse_args()
    shp = [int(v) for v in a.shape.split(",")] if a.shape else None
    if a.op in ("all", "gemm") and a.which != "none":
        for s in ([shp] if shp and a.op == "gemm" else
                  [(16384, 2304, 768), (16384, 768, 768), (16384, 3072, 768), (16384, 768, 3072),
                   (16384, 50257, 768), (8192, 8192, 8192)]):
            bench_gemm(*s, iters=a.iters, cta_group=a.cta_group, which=a.which)
    if a.op in ("all", "attention"):
        for s in ([shp] if shp and a.op == "attention" else [(16, 12, 1024, 64), (8, 25, 1024, 64), (4, 16, 2048, 80), (4, 16, 2048, 128),
                                                               (4, 4, 2048, 128)]):
            bench_attention(*s, iters=a.iters, fwd_only=a.fwd_only)
    if a.op in ("all", "layernorm"):
        for s in ([shp] if shp and a.op == "layernorm" else [(16384, 768), (8192, 4096)]):
            bench_layernorm(*s, iters=a.iters)


if __name__ == "__main__":
    main()
