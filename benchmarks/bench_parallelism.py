#!/usr/bin/env python3
"""Compare data-parallel strategies on one mesh: step time, bytes moved, state and peak memory.

    torchrun --nproc-per-node 8 benchmarks/bench_parallelism.py --precision bf16
    torchrun --nproc-per-node 4 benchmarks/bench_parallelism.py --backend gloo --layers 4 --embd 128

Strategies: ``none``, ``ddp``, ``ddp-no-overlap`` (control for what overlap is
worth), ``fsdp``, ``fsdp-bf16`` (reference benchmarks/bench_parallelism.py).
Communication volume is counted by instrumenting the collectives
(:func:`minidist.record_comm`, which the fused NVLink kernels report into too)
and checked against the analytic prediction; step time is device-timed (CUDA
events, max over ranks) on GPU; ``exposed`` is the share of the step spent in
communication with no compute beside it, from a profiler trace.
"""

from __future__ import annotations

import argparse
import sys
import time
from dataclasses import dataclass, field
from pathlib import Path

import torch

sys.path.insert(0, str(Path(__file__).resolve().parent.parent))

from minidist import (  # noqa: E402
    DistributedDataParallel,
    FullyShardedDataParallel,
    ParallelMesh,
    analyze_trace,
    init_distributed,
    print_rank0,
    profile_steps,
    record_comm,
    resolve_precision,
    shutdown_distributed,
)
from minidist.fsdp import MixedPrecisionPolicy  # noqa: E402
from minidist.models import GPT, Block, GPTConfig  # noqa: E402

STRATEGIES = ["none", "ddp", "ddp-no-overlap", "fsdp", "fsdp-bf16"]


@dataclass
class Row:
    strategy: str
    ms_per_step: float = 0.0
    tokens_per_s: float = 0.0
    comm_bus_mb: float = 0.0
    peak_mem_mb: float = 0.0
    state_mb: float = 0.0
    exposed_comm_pct: float = float("nan")
    per_collective_mb: dict[str, float] = field(default_factory=dict)


def build(strategy, mesh, config, device, cap_mb):
    model = GPT(config, tp_group=mesh.tp_group, device=device)
    if mesh.dp_size == 1 or strategy == "none":
        return model
    if strategy.startswith("ddp"):
        return DistributedDataParallel(model, process_group=mesh.dp_group, bucket_cap_mb=cap_mb,
                                       overlap_with_backward=(strategy == "ddp"))
    pdt = torch.bfloat16 if strategy.endswith("bf16") else torch.float32
    return FullyShardedDataParallel(model, unit_types=(Block,), process_group=mesh.dp_group,
                                    mixed_precision=MixedPrecisionPolicy(param_dtype=pdt, reduce_dtype=torch.float32))


def analytical_comm_mb(strategy: str, config: GPTConfig, mesh: ParallelMesh) -> float:
    """Bus MB per step per rank: DDP 2(W-1)/W*P*4; FSDP (W-1)/W*P*(2*gather_bytes + 4)."""
    w = mesh.dp_size
    if w == 1 or strategy == "none":
        return 0.0
    params = config.param_count() / max(1, mesh.tp_size)
    f = (w - 1) / w
    if strategy.startswith("ddp"):
        return 2 * f * params * 4.0 / 1024**2
    gb = 2.0 if strategy.endswith("bf16") else 4.0
    return f * params * (2 * gb + 4.0) / 1024**2


def measure(strategy, args, mesh, config, device, precision) -> Row:
    torch.manual_seed(args.seed)
    model = build(strategy, mesh, config, device, args.bucket_cap_mb)
    if device.type == "cuda" and all(p.dtype == torch.float32 for p in model.parameters()):
        from minidist.optim import FusedAdamW

        opt = FusedAdamW(model.parameters(), lr=1e-4)
    else:
        opt = torch.optim.AdamW(model.parameters(), lr=1e-4)
    g = torch.Generator().manual_seed(args.seed + mesh.dp_rank)
    ids = torch.randint(0, config.vocab_size, (args.batch_size, config.block_size), generator=g).to(device)
    tgt = torch.randint(0, config.vocab_size, (args.batch_size, config.block_size), generator=g).to(device)

    def step(_=0):
        opt.zero_grad(set_to_none=True)
        with precision.autocast():
            _, loss = model(ids, tgt)
        loss.backward()
        opt.step()

    for _ in range(args.warmup):
        step()
    if device.type == "cuda":
        torch.cuda.synchronize()
        torch.cuda.reset_peak_memory_stats()
    with record_comm() as stats:
        step()
    per = {name: bus / 1024**2 for name, _, _, bus in stats.as_rows()}
    comm_mb = stats.total_bus_bytes() / 1024**2
    if device.type == "cuda":
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        torch.cuda.synchronize()
        a.record()
        for _ in range(args.iters):
            step()
        b.record()
        b.synchronize()
        el = a.elapsed_time(b) / 1e3
    else:
        t0 = time.perf_counter()
        for _ in range(args.iters):
            step()
        el = time.perf_counter() - t0
    t = torch.tensor([el], dtype=torch.float64, device=device)
    if torch.distributed.is_initialized():
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
    el = float(t.item())
    row = Row(strategy, el / args.iters * 1e3, args.batch_size * config.block_size * mesh.dp_size * args.iters / el,
              comm_mb, per_collective_mb=per)
    if device.type == "cuda":
        row.peak_mem_mb = torch.cuda.max_memory_allocated() / 1024**2
    if isinstance(model, FullyShardedDataParallel):
        row.state_mb = model.memory_summary()["fsdp_state_MB"]
    else:
        row.state_mb = sum(p.numel() for p in model.parameters()) * 16 / 1024**2
    if args.profile_dir:
        trace = f"{args.profile_dir}/trace_{strategy}_rank{mesh.rank}.json"
        profile_steps(step, num_steps=6, trace_path=trace)
        if mesh.rank == 0:
            row.exposed_comm_pct = analyze_trace(trace).exposed_fraction_of_step * 100
    return row


def main() -> None:
    p = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    p.add_argument("--tp", type=int, default=1)
    p.add_argument("--strategies", default=",".join(STRATEGIES), type=lambda s: s.split(","))
    p.add_argument("--layers", type=int, default=8)
    p.add_argument("--heads", type=int, default=8)
    p.add_argument("--embd", type=int, default=512)
    p.add_argument("--vocab", type=int, default=8192)
    p.add_argument("--seq-len", type=int, default=256)
    p.add_argument("--batch-size", type=int, default=8)
    p.add_argument("--iters", type=int, default=10)
    p.add_argument("--warmup", type=int, default=3)
    p.add_argument("--bucket-cap-mb", type=float, default=25.0)
    p.add_argument("--seed", type=int, default=1234)
    p.add_argument("--precision", default="fp32", choices=["fp32", "bf16", "auto"])
    p.add_argument("--backend", default=None, choices=[None, "nccl", "gloo"])
    p.add_argument("--profile-dir", default=None)
    args = p.parse_args()

    rank, world, device = init_distributed(backend=args.backend)
    mesh = ParallelMesh(tp_size=args.tp)
    config = GPTConfig(vocab_size=args.vocab, block_size=args.seq_len, n_layer=args.layers, n_head=args.heads,
                       n_embd=args.embd, seed=args.seed)
    precision = resolve_precision(args.precision, device)
    print_rank0(f"\n{'=' * 92}\n  {mesh.describe()}   device={device.type}  precision={precision}")
    print_rank0(f"  model {config.n_layer}L x {config.n_embd}d, vocab {config.vocab_size}, seq {config.block_size}, "
                f"batch {args.batch_size}/replica ({config.param_count() / 1e6:.1f}M params)\n{'=' * 92}")
    print_rank0(f"  {'strategy':<16}{'ms/step':>10}{'tok/s':>12}{'comm MB':>10}{'predicted':>11}"
                f"{'state MB':>10}{'peak MB':>10}{'exposed':>10}\n  " + "-" * 88)
    rows = []
    for s in args.strategies:
        r = measure(s, args, mesh, config, device, precision)
        rows.append(r)
        exposed = "-" if r.exposed_comm_pct != r.exposed_comm_pct else f"{r.exposed_comm_pct:.1f}%"
        print_rank0(f"  {s:<16}{r.ms_per_step:>10.2f}{r.tokens_per_s:>12.0f}{r.comm_bus_mb:>10.1f}"
                    f"{analytical_comm_mb(s, config, mesh):>11.1f}{r.state_mb:>10.1f}{r.peak_mem_mb:>10.1f}{exposed:>10}")
    print_rank0("\n  per-collective bus traffic (MB/step/rank):")
    for r in rows:
        if r.per_collective_mb:
            print_rank0(f"    {r.strategy:<16}" + "  ".join(f"{k}={v:.1f}" for k, v in sorted(r.per_collective_mb.items())))
    base = next((r for r in rows if r.strategy == "ddp"), None)
    if base and len(rows) > 1:
        print_rank0("\n  relative to ddp:")
        for r in rows:
            if r is not base:
                print_rank0(f"    {r.strategy:<16}{base.ms_per_step / r.ms_per_step:>6.2f}x speed   "
                            f"{r.comm_bus_mb / max(base.comm_bus_mb, 1e-9):>5.2f}x comm   "
                            f"{r.state_mb / max(base.state_mb, 1e-9):>5.2f}x state")
    shutdown_distributed()


if __name__ == "__main__":
    main()
