#!/usr/bin/env python3
"""Collective microbenchmark: NCCL all-reduce / all-gather / reduce-scatter / broadcast,
plus this framework's peer-memory all-reduce kernel where available.

    torchrun --nproc-per-node 8 benchmarks/bench_collectives.py --max-mb 256

Reports algorithm bandwidth (payload / time) and bus bandwidth (bytes that
cross the interconnect / time; all-reduce 2(W-1)/W * S, all-gather and
reduce-scatter (W-1)/W * S, broadcast S), each as the slowest rank's average
(reference benchmarks/bench_collectives.py:1-30, 71-89).  Times are CUDA-event
device times on GPU.  The ``md_allreduce`` rows run the fused kernel of
csrc/symm.cu on fp32 buffers in symmetric memory (the DDP bucket path).
"""

from __future__ import annotations

import argparse
import csv
import sys
import time
from dataclasses import dataclass
from pathlib import Path

import torch
import torch.distributed as dist

sys.path.insert(0, str(Path(__file__).resolve().parent.parent))

from minidist import init_distributed, print_rank0, shutdown_distributed  # noqa: E402


@dataclass
class Result:
    collective: str
    payload_bytes: int
    seconds: float
    bus_bytes: float

    @property
    def alg_gbps(self) -> float:
        return self.payload_bytes / self.seconds / 1e9

    @property
    def bus_gbps(self) -> float:
        return self.bus_bytes / self.seconds / 1e9


def time_op(fn, device, iters: int, warmup: int) -> float:
    for _ in range(warmup):
        fn()
    if device.type == "cuda":
        torch.cuda.synchronize()
    dist.barrier()
    if device.type == "cuda":
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        for _ in range(iters):
            fn()
        b.record()
        b.synchronize()
        sec = a.elapsed_time(b) / 1e3 / iters
    else:
        t0 = time.perf_counter()
        for _ in range(iters):
            fn()
        sec = (time.perf_counter() - t0) / iters
    t = torch.tensor([sec], device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def run(args) -> list[Result]:
    rank, world, device = init_distributed(backend=args.backend)
    dtype = {"fp32": torch.float32, "bf16": torch.bfloat16, "fp16": torch.float16}[args.dtype]
    item = torch.empty((), dtype=dtype).element_size()
    fused = None
    if device.type == "cuda" and "md_allreduce" in args.collectives:
        from minidist.parallel import collectives, symm

        c = symm.communicator(None, list(range(world)))
        if c is not None:
            fused = (collectives, symm, c, symm.SymmBuffer(None, args.max_mb * 1024 * 1024 + 4096))
    print_rank0(f"\n{'=' * 78}\n  collective microbenchmark   world={world}  backend={dist.get_backend()}  "
                f"dtype={args.dtype}  device={device.type}\n{'=' * 78}")
    print_rank0(f"  {'collective':<16}{'size (MB)':>12}{'time (ms)':>12}{'algbw GB/s':>12}{'busbw GB/s':>12}")
    results: list[Result] = []
    size = args.min_kb * 1024
    while size <= args.max_mb * 1024 * 1024:
        numel = (size // item) // (world * 64) * (world * 64)
        if numel == 0:
            size *= 2
            continue
        payload = numel * item
        buf = torch.ones(numel, dtype=dtype, device=device)
        shard = torch.ones(numel // world, dtype=dtype, device=device)
        specs = [
            ("all_reduce", lambda b=buf: dist.all_reduce(b), 2 * (world - 1) / world * payload),
            ("all_gather", lambda b=buf, s=shard: dist.all_gather_into_tensor(b, s), (world - 1) / world * payload),
            ("reduce_scatter", lambda b=buf, s=shard: dist.reduce_scatter_tensor(s, b), (world - 1) / world * payload),
            ("broadcast", lambda b=buf: dist.broadcast(b, src=0), float(payload)),
        ]
        if fused is not None:
            coll, _, comm_, sbuf = fused
            n32 = (numel * item // 4) // 64 * 64
            specs.append(("md_allreduce", lambda n=n32: coll.allreduce_fp32_(sbuf, comm_, 0, n, 1.0, 2),
                          2 * (world - 1) / world * n32 * 4))
        for name, fn, bus in specs:
            if name not in args.collectives:
                continue
            sec = time_op(fn, device, args.iters, args.warmup)
            pb = payload if name != "md_allreduce" else (numel * item // 4) // 64 * 64 * 4
            r = Result(name, pb, sec, bus)
            results.append(r)
            print_rank0(f"  {name:<16}{pb / 1024**2:>12.2f}{sec * 1e3:>12.3f}{r.alg_gbps:>12.2f}{r.bus_gbps:>12.2f}")
        size *= 2
    if args.csv and rank == 0:
        with open(args.csv, "w", newline="") as fh:
            w = csv.writer(fh)
            w.writerow(["collective", "world_size", "payload_bytes", "seconds", "alg_gbps", "bus_gbps"])
            for r in results:
                w.writerow([r.collective, world, r.payload_bytes, f"{r.seconds:.9f}", f"{r.alg_gbps:.4f}",
                            f"{r.bus_gbps:.4f}"])
        print_rank0(f"\n  wrote {args.csv}")
    shutdown_distributed()
    return results


def main() -> None:
    p = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    p.add_argument("--min-kb", type=int, default=64)
    p.add_argument("--max-mb", type=int, default=128)
    p.add_argument("--iters", type=int, default=20)
    p.add_argument("--warmup", type=int, default=5)
    p.add_argument("--dtype", default="fp32", choices=["fp32", "bf16", "fp16"])
    p.add_argument("--backend", default=None, choices=[None, "nccl", "gloo"])
    p.add_argument("--csv", default=None)
    p.add_argument("--collectives", default="all_reduce,all_gather,reduce_scatter,broadcast,md_allreduce",
                   type=lambda s: s.split(","))
    run(p.parse_args())


if __name__ == "__main__":
    main()
