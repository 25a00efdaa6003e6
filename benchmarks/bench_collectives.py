#!/usr/bin/env python3
"""Collective bandwidth: NCCL's collectives beside this framework's peer-memory kernels.

    torchrun --nproc-per-node 8 benchmarks/bench_collectives.py --max-mb 1024
    torchrun --nproc-per-node 8 benchmarks/bench_collectives.py --ops nccl_all_reduce,md_ar_bucket --json bw.jsonl

Each op is an :class:`Op` -- how to build its buffers for a payload, the call,
and its bus-byte factor (bytes that cross the interconnect per rank, per
payload byte: all-reduce 2(W-1)/W, all-gather / reduce-scatter (W-1)/W,
broadcast 1; the reference's accounting, benchmarks/bench_collectives.py).
Ops:

* ``nccl_all_reduce``, ``nccl_all_gather``, ``nccl_reduce_scatter``,
  ``nccl_broadcast`` -- torch.distributed (NCCL on GPUs, Gloo on CPU);
* ``md_ar_bucket`` -- the DDP gradient all-reduce kernel (fp32, symmetric
  memory, 1/W scale fused);
* ``md_ag_shards`` -- the FSDP parameter gather kernel (fp32 shards gathered
  and cast to bf16 in one pass; payload = the bf16 output);
* ``md_rs_shard`` -- the FSDP gradient reduce-scatter kernel (fp32).

Payloads grow geometrically from ``--min-kb`` to ``--max-mb`` by ``--factor``.
Time per call is the slowest rank's CUDA-event average after warm-up.  The
printout is one row per payload and one bus-GB/s column per op.
"""

from __future__ import annotations

import argparse
import json
import sys
import time
from collections.abc import Callable
from dataclasses import dataclass
from pathlib import Path

import torch
import torch.distributed as dist

sys.path.insert(0, str(Path(__file__).resolve().parent.parent))

from minidist import init_distributed, print_rank0, shutdown_distributed  # noqa: E402


@dataclass(frozen=True)
class Op:
    name: str
    bus_factor: Callable[[int], float]     # world -> bus bytes per payload byte
    build: Callable[[int, dict], Callable]  # (payload bytes, context) -> call
    native: bool = False                   # needs the peer-memory runtime (CUDA, one node)


def _nccl(kind: str):
    def build(nbytes: int, ctx: dict):
        w, dev, dt = ctx["world"], ctx["device"], ctx["dtype"]
        n = max(w, nbytes // dt.itemsize // w * w)
        full = torch.ones(n, dtype=dt, device=dev)
        part = torch.ones(n // w, dtype=dt, device=dev)
        return {
            "all_reduce": lambda: dist.all_reduce(full),
            "all_gather": lambda: dist.all_gather_into_tensor(full, part),
            "reduce_scatter": lambda: dist.reduce_scatter_tensor(part, full),
            "broadcast": lambda: dist.broadcast(full, src=0),
        }[kind]
    return build


def _symm(ctx: dict, nbytes: int):
    """A symmetric buffer of at least ``nbytes`` shared by the native ops (grown on demand)."""
    from minidist.parallel import symm

    c = symm.communicator(None, list(range(ctx["world"])))
    return c, c.buffer("bench_collectives", nbytes + 4096)


def _md_ar(nbytes: int, ctx: dict):
    from minidist.parallel import collectives

    c, buf = _symm(ctx, nbytes)
    n = max(64, nbytes // 4 // 64 * 64)
    return lambda: collectives.allreduce_fp32_(buf, c, 0, n, 1.0 / c.world, 2)


def _md_ag(nbytes: int, ctx: dict):
    from minidist.parallel import collectives

    w = ctx["world"]
    shard = max(4, nbytes // 2 // w // 4 * 4)  # payload = the bf16 gathered output
    c, buf = _symm(ctx, shard * 4)
    out = torch.empty(shard * w, dtype=torch.bfloat16, device=ctx["device"])
    return lambda: collectives.all_gather_shards(buf, c, 0, shard, out)


def _md_rs(nbytes: int, ctx: dict):
    from minidist.parallel import collectives

    w = ctx["world"]
    shard = max(4, nbytes // 4 // w // 4 * 4)
    c, buf = _symm(ctx, shard * w * 4)
    grad = torch.empty(shard, dtype=torch.float32, device=ctx["device"])
    return lambda: collectives.reduce_scatter_shard(buf, c, 0, shard, grad, False, 1.0 / w)


OPS: dict[str, Op] = {op.name: op for op in (
    Op("nccl_all_reduce", lambda w: 2 * (w - 1) / w, _nccl("all_reduce")),
    Op("nccl_all_gather", lambda w: (w - 1) / w, _nccl("all_gather")),
    Op("nccl_reduce_scatter", lambda w: (w - 1) / w, _nccl("reduce_scatter")),
    Op("nccl_broadcast", lambda w: 1.0, _nccl("broadcast")),
    Op("md_ar_bucket", lambda w: 2 * (w - 1) / w, _md_ar, native=True),
    Op("md_ag_shards", lambda w: (w - 1) / w, _md_ag, native=True),
    Op("md_rs_shard", lambda w: (w - 1) / w, _md_rs, native=True),
)}


def seconds_per_call(fn: Callable, device, iters: int, warmup: int) -> float:
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
    t = torch.tensor([sec], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def main(argv=None) -> list[dict]:
    p = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    p.add_argument("--ops", default=",".join(OPS), type=lambda v: v.split(","))
    p.add_argument("--min-kb", type=int, default=256)
    p.add_argument("--max-mb", type=int, default=256)
    p.add_argument("--factor", type=int, default=4)
    p.add_argument("--iters", type=int, default=20)
    p.add_argument("--warmup", type=int, default=5)
    p.add_argument("--dtype", default="fp32", choices=["fp32", "bf16"], help="dtype of the NCCL ops")
    p.add_argument("--backend", default=None, choices=[None, "nccl", "gloo"])
    p.add_argument("--json", default=None, metavar="PATH", help="rank 0 appends one record per (op, payload)")
    args = p.parse_args(argv)
    rank, world, device = init_distributed(backend=args.backend)
    ctx = {"world": world, "device": device, "dtype": {"fp32": torch.float32, "bf16": torch.bfloat16}[args.dtype]}
    native_ok = False
    if device.type == "cuda":
        from minidist.parallel import symm

        native_ok = symm.communicator(None, list(range(world))) is not None
    ops = [OPS[o] for o in args.ops if o in OPS and (native_ok or not OPS[o].native)]
    skipped = [o for o in args.ops if o not in [op.name for op in ops]]
    print_rank0(f"\ncollective bus bandwidth (GB/s), world {world}, {dist.get_backend()} on {device.type}"
                + (f"; skipped {skipped} (no peer-memory runtime here)" if skipped else ""))
    print_rank0(f"{'payload':>10}" + "".join(f"{op.name:>21}" for op in ops))
    records = []
    size = args.min_kb * 1024
    while size <= args.max_mb * 2**20:
        cells = []
        for op in ops:
            sec = seconds_per_call(op.build(size, ctx), device, args.iters, args.warmup)
            bus = op.bus_factor(world) * size
            cells.append(f"{bus / sec / 1e9:>13.1f} ({sec * 1e6:>5.0f}us)")
            records.append(dict(op=op.name, world=world, payload_bytes=size, us=sec * 1e6,
                                bus_gbps=bus / sec / 1e9, alg_gbps=size / sec / 1e9))
        label = f"{size / 2**20:.2f} MB" if size >= 2**20 else f"{size // 1024} KB"
        print_rank0(f"{label:>10}" + "".join(f"{c:>21}" for c in cells))
        size *= args.factor
    if args.json and rank == 0:
        with open(args.json, "a") as fh:
            for r in records:
                fh.write(json.dumps(r) + "\n")
    shutdown_distributed()
    return records


if __name__ == "__main__":
    main()
