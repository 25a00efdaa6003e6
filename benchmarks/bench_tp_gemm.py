#!/usr/bin/env python3
"""Row-parallel linear with its all-reduce: fused kernel vs GEMM + NCCL.

    torchrun --nproc-per-node 8 --master-addr 127.0.0.1 benchmarks/bench_tp_gemm.py
    torchrun --nproc-per-node 8 --master-addr 127.0.0.1 benchmarks/bench_tp_gemm.py --sweep baseline

For each shape (M tokens, K = input features per rank, N = output features)
it times, on the device (CUDA events, max over ranks, after warm-up):

* ``fused``  — ``md_gemm_ar``: one persistent kernel; the GEMM epilogue
  publishes bf16 partial tiles in symmetric memory and comm warps of the same
  kernel reduce this rank's tiles over NVLink (bias + residual added once) and
  copy the rest from their owners;
* ``nccl``   — our tcgen05 GEMM, then NCCL all-reduce of the bf16 output,
  then bias and residual;
* ``ref``    — the reference's row-parallel linear itself
  (tensor_parallel.py:351-358, under bf16 autocast): ``F.linear`` (cuBLAS),
  ``all_reduce`` over NCCL, bias added after the reduce, then the residual add
  of its block (models/gpt.py:163-166).

The roofline column is max(GEMM FLOPs / measured bf16 peak, NVLink bytes per
rank / 770 GB/s), with NVLink bytes = 2 (W-1)/W * M * N * 2 (the all-reduce
bus bytes); ``frac`` = roofline time / measured time.
"""

from __future__ import annotations

import argparse
import json
import os
import sys
from pathlib import Path

import torch
import torch.distributed as dist

sys.path.insert(0, str(Path(__file__).resolve().parent.parent))

from minidist import init_distributed, print_rank0, shutdown_distributed  # noqa: E402
from minidist.parallel import collectives  # noqa: E402

SHAPES = [  # (M, K per rank at tp=8, N): GPT-2 small attn.proj / mlp.proj, 6.7B attn.proj / mlp.proj
    (16384, 96, 768),
    (16384, 384, 768),
    (8192, 512, 4096),
    (8192, 2048, 4096),
]


def _peak_tflops() -> float:
    f = Path(__file__).resolve().parent.parent / "MEASURED_PEAKS.json"
    try:
        return float(json.loads(f.read_text())["bf16_tflops"])
    except Exception:
        return 1590.0


def timed(fn, iters: int, warmup: int) -> tuple[float, float]:
    """(device seconds per call, host seconds per call), each the max over ranks."""
    import time

    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    dist.barrier()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    h0 = time.perf_counter()
    for _ in range(iters):
        fn()
    h1 = time.perf_counter()
    b.record()
    b.synchronize()
    t = torch.tensor([a.elapsed_time(b) / iters / 1e3, (h1 - h0) / iters], device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t[0].item()), float(t[1].item())


def main() -> None:
    p = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    p.add_argument("--iters", type=int, default=20)
    p.add_argument("--warmup", type=int, default=5)
    p.add_argument("--json", metavar="PATH", default=None, help="rank 0 appends one JSON line per shape")
    p.add_argument("--sweep", default="gpt", choices=["gpt", "baseline"],
                   help="gpt: GPT-2 small / 6.7B layer shapes (K per rank as at tp=8); "
                        "baseline: M in {2048, 8192, 32768}, K = N = 4096 (K split over the ranks)")
    args = p.parse_args()
    rank, world, device = init_distributed(backend="nccl")
    peak = _peak_tflops() * 1e12
    print_rank0(f"\n  row-parallel GEMM + all-reduce, W={world}  (times: max over ranks)")
    print_rank0(f"  {'M':>6}{'K':>6}{'N':>6}{'fused us':>10}{'nccl us':>10}{'ref us':>10}{'vs ref':>8}"
                f"{'roofline us':>13}{'frac':>7}{'host us (fused/nccl)':>22}")
    if args.sweep == "baseline":
        shapes = [(M, 4096 // world, 4096) for M in (2048, 8192, 32768)]
    else:
        shapes = [(M, max(64, K8 * 8 // world), N) for M, K8, N in SHAPES]
    for M, K, N in shapes:
        g = torch.Generator(device="cuda").manual_seed(rank)
        x = torch.randn(M, K, device="cuda", generator=g).bfloat16()
        w = (torch.randn(N, K, device="cuda", generator=g) * 0.05).bfloat16()
        bias = torch.randn(N, device="cuda", generator=g)
        resid = torch.randn(M, N, device="cuda", generator=g).bfloat16()
        os.environ["MINIDIST_TP_FUSED"] = "1"
        tf, hf = timed(lambda: collectives.gemm_all_reduce(x, w, bias, resid, None), args.iters, args.warmup)
        os.environ["MINIDIST_TP_FUSED"] = "0"
        tn, hn = timed(lambda: collectives.gemm_all_reduce(x, w, bias, resid, None), args.iters, args.warmup)
        os.environ["MINIDIST_TP_FUSED"] = "1"

        def reference_row_parallel():
            with torch.autocast("cuda", dtype=torch.bfloat16):
                y = torch.nn.functional.linear(x, w)
                dist.all_reduce(y)
                y = y + bias
                return resid + y

        tr, _ = timed(reference_row_parallel, args.iters, args.warmup)
        flops = 2.0 * M * N * K
        nv = 2.0 * (world - 1) / world * M * N * 2
        roof = max(flops / peak, nv / 770e9)
        print_rank0(f"  {M:>6}{K:>6}{N:>6}{tf * 1e6:>10.1f}{tn * 1e6:>10.1f}{tr * 1e6:>10.1f}{tr / tf:>7.2f}x"
                    f"{roof * 1e6:>13.1f}{roof / tf:>7.2f}{hf * 1e6:>12.1f}/{hn * 1e6:.1f}")
        if args.json and rank == 0:
            with open(args.json, "a") as f:
                f.write(json.dumps(dict(world=world, M=M, K=K, N=N, fused_us=tf * 1e6, nccl_us=tn * 1e6,
                                        ref_us=tr * 1e6, roofline_us=roof * 1e6, frac=roof / tf)) + "\n")
    shutdown_distributed()


if __name__ == "__main__":
    main()
