#!/usr/bin/env python3
"""Single-GPU driver of the fused collective kernels, for ncu captures.

    python benchmarks/fused_kernels_1gpu.py --kernel gemm_ar --iters 3
    python benchmarks/fused_kernels_1gpu.py --kernel ddp_ar --iters 3
    python benchmarks/fused_kernels_1gpu.py --kernel fsdp_rs --iters 3
    python benchmarks/fused_kernels_1gpu.py --kernel fsdp_ag --iters 3

ncu profiles one process on one GPU, so this runs each kernel with a group of
one rank on ordinary device buffers (every "peer" pointer is this rank's own
buffer): the GEMM, epilogue, staging and memory structure are the real
kernels'; the NVLink side is measured on several GPUs by
benchmarks/bench_tp_gemm.py and benchmarks/bench_collectives.py.

* ``gemm_ar``  -- md_gemm_ar (GEMM + tensor-parallel all-reduce), M=8192,
  K=512, N=4096 (the 6.7B attention projection at tp=8), bias + residual.
* ``ddp_ar``   -- md_ar_bucket_kernel on a 25 MB fp32 bucket (1/W scale).
* ``fsdp_rs``  -- md_rs_shard_kernel with the in-kernel AdamW on a 40 M-element shard.
* ``fsdp_ag``  -- md_ag_shards_kernel: a 40 M-element fp32 shard gathered as bf16.
* ``fsdp_ag_bf16`` -- md_ag_shards_kernel on bf16 shard copies (the bf16-gather path).
* ``ce_tp``    -- md_ce_tp_kernel: the vocab-parallel cross-entropy statistics of
  8192 tokens over 50304 / 8 columns (50 slabs of 128).
* ``embed_tp`` -- md_embed_tp_kernel: 8192 token rows of 4096 bf16 gathered from
  the (here local) shard that owns them, positions added.
"""

from __future__ import annotations

import argparse
import ctypes
import sys
from pathlib import Path

import torch

sys.path.insert(0, str(Path(__file__).resolve().parent.parent))

from minidist.ops import _native as nat  # noqa: E402
from minidist.ops import gemm as G  # noqa: E402
from minidist.parallel import collectives as C  # noqa: E402


def timed(fn, iters: int) -> float:
    for _ in range(3):
        fn()
    torch.cuda.synchronize()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    for _ in range(iters):
        fn()
    b.record()
    b.synchronize()
    return a.elapsed_time(b) / iters / 1e3


def run_gemm_ar(iters: int) -> None:
    M, K, N = 8192, 512, 4096
    x = torch.randn(M, K, device="cuda").bfloat16()
    w = (torch.randn(N, K, device="cuda") * 0.05).bfloat16()
    bias = torch.randn(N, device="cuda")
    resid = torch.randn(M, N, device="cuda").bfloat16()
    part = torch.empty(M, N, dtype=torch.bfloat16, device="cuda")
    fin = torch.empty_like(part)
    chunks = (M + 31) // 32 * ((N + 255) // 256)
    flags = torch.zeros(2 * chunks, dtype=torch.int32, device="cuda")
    out = torch.empty(M, N, dtype=torch.bfloat16, device="cuda")
    ar = C.TpArParams()
    ar.partial[0], ar.fin[0], ar.flags[0] = part.data_ptr(), fin.data_ptr(), flags.data_ptr()
    ar.ldp, ar.out, ar.ldo = N, out.data_ptr(), N
    ar.bias, ar.resid, ar.ldr = bias.data_ptr(), resid.data_ptr(), N
    ar.world, ar.rank, ar.max_chunks, ar.timeout_ns = 1, 0, chunks, 10**10
    claim = torch.zeros(3, dtype=torch.int32, device="cuda")
    ar.claim = claim.data_ptr()
    gp = nat.GemmParams()
    gp.A, gp.B, gp.lda, gp.ldb = x.data_ptr(), w.data_ptr(), K, K
    gp.M, gp.N, gp.K, gp.epi, gp.alpha = M, N, K, G.EPI_BF16, 1.0
    gp.status = nat.status_ptr()
    def call():
        nat.check(nat.lib().md_gemm_ar(ctypes.byref(gp), ctypes.byref(ar), ctypes.c_void_p(nat.stream_ptr())),
                  "md_gemm_ar")

    t = timed(call, iters)
    nat.check_status()
    want = (x.float() @ w.float().t() + bias + resid.float())
    err = ((out.float() - want).abs().max() / want.abs().max()).item()
    assert claim.tolist()[:2] == [0, 0], "cluster-order counters not reset"
    print(f"md_gemm_ar world=1 M={M} K={K} N={N}: {t * 1e6:.1f} us, {2 * M * N * K / t / 1e12:.0f} TFLOP/s, "
          f"rel err {err:.2e}")


def run_ddp_ar(iters: int) -> None:
    n = 25 * 1024 * 1024 // 4 // 64 * 64
    buf = torch.randn(n, device="cuda")
    flags = torch.zeros(int(nat.lib().md_symm_flag_bytes()) // 4, dtype=torch.int32, device="cuda")
    p = C.ArParams()
    p.bufs[0], p.flags[0] = buf.data_ptr(), flags.data_ptr()
    p.offset, p.n, p.world, p.rank, p.scale, p.channel = 0, n, 1, 0, 1.0, 0
    p.timeout_ns, p.status = 10**10, nat.status_ptr()
    ctas = nat.lib().md_allreduce_ctas(n, 1)
    def call():
        nat.check(nat.lib().md_allreduce(ctypes.byref(p), ctas, ctypes.c_void_p(nat.stream_ptr())), "md_allreduce")

    t = timed(call, iters)
    nat.check_status()
    print(f"md_ar_bucket world=1 25 MB: {t * 1e6:.1f} us, {2 * n * 4 / t / 1e9:.0f} GB/s (read + write)")


def run_fsdp_rs(iters: int) -> None:
    shard = 40 * 1024 * 1024
    grads = torch.randn(shard, device="cuda")
    flags = torch.zeros(int(nat.lib().md_symm_flag_bytes()) // 4, dtype=torch.int32, device="cuda")
    pmv = [torch.randn(shard, device="cuda") for _ in range(2)] + [torch.rand(shard, device="cuda")]
    r = C.RsParams()
    r.bufs[0], r.flags[0] = grads.data_ptr(), flags.data_ptr()
    r.offset, r.shard, r.world, r.rank, r.scale, r.channel = 0, shard, 1, 0, 1.0, 4
    r.timeout_ns, r.status = 10**10, nat.status_ptr()
    r.p, r.m, r.v = (t.data_ptr() for t in pmv)
    r.lr, r.b1, r.b2, r.eps, r.wd, r.bc1, r.bc2_sqrt = 1e-4, 0.9, 0.999, 1e-8, 0.01, 0.1, 0.0316
    def call():
        nat.check(nat.lib().md_rs_shard(ctypes.byref(r), nat.num_sms(), ctypes.c_void_p(nat.stream_ptr())), "md_rs_shard")

    t = timed(call, iters)
    nat.check_status()
    print(f"md_rs_shard+AdamW world=1 {shard / 1e6:.0f} M elements: {t * 1e6:.1f} us, "
          f"{7 * shard * 4 / t / 1e9:.0f} GB/s (g, p, m, v read + p, m, v write)")


def run_fsdp_ag(iters: int) -> None:
    shard = 40 * 1024 * 1024
    src = torch.randn(shard, device="cuda")
    out = torch.empty(shard, dtype=torch.bfloat16, device="cuda")
    flags = torch.zeros(int(nat.lib().md_symm_flag_bytes()) // 4, dtype=torch.int32, device="cuda")
    a = C.AgParams()
    a.bufs[0], a.flags[0] = src.data_ptr(), flags.data_ptr()
    a.offset, a.shard, a.world, a.rank, a.channel = 0, shard, 1, 0, 5
    a.timeout_ns, a.status = 10**10, nat.status_ptr()
    a.out, a.out_bf16 = out.data_ptr(), 1
    def call():
        nat.check(nat.lib().md_ag_shards(ctypes.byref(a), 64, ctypes.c_void_p(nat.stream_ptr())), "md_ag_shards")

    t = timed(call, iters)
    nat.check_status()
    assert torch.equal(out, src.bfloat16())
    print(f"md_ag_shards world=1 {shard / 1e6:.0f} M elements fp32->bf16: {t * 1e6:.1f} us, "
          f"{6 * shard / t / 1e9:.0f} GB/s (read + write)")


def run_fsdp_ag_bf16(iters: int) -> None:
    shard = 40 * 1024 * 1024
    src = torch.randn(shard, device="cuda").bfloat16()
    out = torch.empty(shard, dtype=torch.bfloat16, device="cuda")
    flags = torch.zeros(int(nat.lib().md_symm_flag_bytes()) // 4, dtype=torch.int32, device="cuda")
    a = C.AgParams()
    a.bufs[0], a.flags[0] = src.data_ptr(), flags.data_ptr()
    a.offset, a.shard, a.world, a.rank, a.channel = 0, shard, 1, 0, 5
    a.timeout_ns, a.status = 10**10, nat.status_ptr()
    a.out, a.out_bf16, a.in_bf16 = out.data_ptr(), 1, 1
    def call():
        nat.check(nat.lib().md_ag_shards(ctypes.byref(a), 64, ctypes.c_void_p(nat.stream_ptr())), "md_ag_shards")

    t = timed(call, iters)
    nat.check_status()
    assert torch.equal(out, src)
    print(f"md_ag_shards world=1 {shard / 1e6:.0f} M elements bf16->bf16: {t * 1e6:.1f} us, "
          f"{4 * shard / t / 1e9:.0f} GB/s (read + write)")


def run_ce_tp(iters: int) -> None:
    M, tiles = 8192, -(-50304 // 8 // 128)
    tmax = torch.randn(tiles, M, device="cuda")
    tsum = torch.rand(tiles, M, device="cuda") * 100
    ttgt = torch.randn(M, device="cuda")
    buf = torch.empty(3 * M, device="cuda")
    flags = torch.zeros(int(nat.lib().md_symm_flag_bytes()) // 4, dtype=torch.int32, device="cuda")
    lse, loss = torch.empty(M, device="cuda"), torch.empty(M, device="cuda")
    prm = C.CeTpParams()
    prm.bufs[0], prm.flags[0] = buf.data_ptr(), flags.data_ptr()
    prm.world, prm.rank, prm.channel = 1, 0, 6
    prm.timeout_ns, prm.status = 10**10, nat.status_ptr()
    prm.tmax, prm.tsum, prm.tiles, prm.ttgt, prm.M = tmax.data_ptr(), tsum.data_ptr(), tiles, ttgt.data_ptr(), M
    prm.lse, prm.loss = lse.data_ptr(), loss.data_ptr()
    ctas = min(64, max(1, -(-M // 256)))
    def call():
        nat.check(nat.lib().md_ce_tp(ctypes.byref(prm), ctas, ctypes.c_void_p(nat.stream_ptr())), "md_ce_tp")

    t = timed(call, iters)
    nat.check_status()
    want = torch.logsumexp(tmax + torch.log(tsum), 0)
    assert (lse - want).abs().max().item() < 1e-3
    print(f"md_ce_tp world=1 M={M} tiles={tiles}: {t * 1e6:.1f} us, "
          f"{(2 * tiles + 1 + 5) * M * 4 / t / 1e9:.0f} GB/s")


def run_embed_tp(iters: int) -> None:
    V, C_, M, S = 50304 // 8, 4096, 8192, 2048
    wte = torch.randn(V, C_, device="cuda").bfloat16()
    wpe = torch.randn(S, C_, device="cuda").bfloat16()
    ids = torch.randint(0, V, (M,), device="cuda")
    out = torch.empty(M, C_, dtype=torch.bfloat16, device="cuda")
    flags = torch.zeros(int(nat.lib().md_symm_flag_bytes()) // 4, dtype=torch.int32, device="cuda")
    prm = C.EmbTpParams()
    prm.wte[0], prm.flags[0] = wte.data_ptr(), flags.data_ptr()
    prm.world, prm.rank, prm.channel = 1, 0, 7
    prm.timeout_ns, prm.status = 10**10, nat.status_ptr()
    prm.ids, prm.wpe, prm.ldp, prm.out, prm.ldo = ids.data_ptr(), wpe.data_ptr(), C_, out.data_ptr(), C_
    prm.ldw, prm.vocab_rows, prm.M, prm.S, prm.C = C_, V, M, S, C_
    ctas = min(148, max(1, -(-M // 32)))
    def call():
        nat.check(nat.lib().md_embed_tp(ctypes.byref(prm), ctas, ctypes.c_void_p(nat.stream_ptr())), "md_embed_tp")

    t = timed(call, iters)
    nat.check_status()
    want = (wte.float()[ids] + wpe.float()[torch.arange(M, device="cuda") % S]).bfloat16()
    assert torch.equal(out, want)
    print(f"md_embed_tp world=1 {M} rows x {C_}: {t * 1e6:.1f} us, {3 * M * C_ * 2 / t / 1e9:.0f} GB/s")


def main() -> None:
    a = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    a.add_argument("--kernel", default="all", choices=["all", "gemm_ar", "ddp_ar", "fsdp_rs", "fsdp_ag",
                                                       "fsdp_ag_bf16", "ce_tp", "embed_tp"])
    a.add_argument("--iters", type=int, default=20)
    args = a.parse_args()
    if args.kernel in ("all", "gemm_ar"):
        run_gemm_ar(args.iters)
    if args.kernel in ("all", "ddp_ar"):
        run_ddp_ar(args.iters)
    if args.kernel in ("all", "fsdp_rs"):
        run_fsdp_rs(args.iters)
    if args.kernel in ("all", "fsdp_ag"):
        run_fsdp_ag(args.iters)
    if args.kernel in ("all", "fsdp_ag_bf16"):
        run_fsdp_ag_bf16(args.iters)
    if args.kernel in ("all", "ce_tp"):
        run_ce_tp(args.iters)
    if args.kernel in ("all", "embed_tp"):
        run_embed_tp(args.iters)


if __name__ == "__main__":
    main()
