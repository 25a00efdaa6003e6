#!/usr/bin/env python3
"""Data-parallel strategies side by side: step time, bus traffic, memory, and where the time went.

    torchrun --nproc-per-node 8 benchmarks/bench_parallelism.py --precision bf16
    torchrun --nproc-per-node 8 benchmarks/bench_parallelism.py --precision bf16 --strategies ddp,ddp-nccl --trace-dir tr
    torchrun --nproc-per-node 4 benchmarks/bench_parallelism.py --backend gloo --layers 4 --embd 128

Each strategy is a :class:`Strategy`: how to wrap the model, which collective
path it forces, and its analytic bus bytes per step and rank (the reference's
accounting, benchmarks/bench_parallelism.py:87-105: DDP all-reduces fp32
gradients, ``2(W-1)/W * 4P``; ZeRO-3 gathers parameters twice in the gather
dtype and reduce-scatters fp32 gradients, ``(W-1)/W * P * (2 g + 4)``).

Strategies: ``none``, ``ddp`` (peer-memory bucket all-reduce on CUDA),
``ddp-nccl`` (the same buckets through NCCL), ``ddp-no-overlap`` (all buckets
after backward), ``fsdp``, ``fsdp-bf16``, ``fsdp-bf16-nccl`` (gathers and
reduce-scatters through NCCL) and ``fsdp-bf16-adamw`` (AdamW applied to each
shard inside the reduce-scatter kernel).  On Gloo/CPU the ``-nccl`` variants
equal their base strategy.

Per strategy, on every rank: K device-timed steps (CUDA events, the maximum
over ranks), one instrumented step whose collectives report their bus bytes
(:func:`minidist.record_comm`; the fused kernels report with the same
formulas), and with ``--trace-dir`` a profiled window whose trace gives the
exposed-communication and fused-kernel shares of the step plus, on CUDA, the
fused kernels' device-side peer-wait share (:class:`minidist.profiling.PeerWaitCounters`).
``--json`` appends one record per strategy.
"""

from __future__ import annotations

import argparse
import json
import os
import sys
import time
from collections.abc import Callable
from dataclasses import asdict, dataclass, field
from pathlib import Path

import torch
import torch.distributed as dist

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


@dataclass(frozen=True)
class Strategy:
    name: str
    kind: str                      # "none" | "ddp" | "fsdp"
    overlap: bool = True           # DDP: buckets launched during backward
    gather_dtype: torch.dtype = torch.float32
    env: tuple[tuple[str, str], ...] = ()   # collective-path switches read at construction
    adamw_in_kernel: bool = False

    def bus_mb(self, params: float, world: int) -> float:
        if world == 1 or self.kind == "none":
            return 0.0
        frac = (world - 1) / world
        if self.kind == "ddp":
            return 2 * frac * params * 4 / 2**20
        g = torch.finfo(self.gather_dtype).bits / 8
        return frac * params * (2 * g + 4) / 2**20


_NCCL = (("MINIDIST_DDP_REDUCER", "nccl"), ("MINIDIST_FSDP_FUSED", "0"), ("MINIDIST_FSDP_GATHER", "0"))
STRATEGIES: dict[str, Strategy] = {s.name: s for s in (
    Strategy("none", "none"),
    Strategy("ddp", "ddp"),
    Strategy("ddp-nccl", "ddp", env=_NCCL),
    Strategy("ddp-no-overlap", "ddp", overlap=False),
    Strategy("fsdp", "fsdp"),
    Strategy("fsdp-bf16", "fsdp", gather_dtype=torch.bfloat16),
    Strategy("fsdp-bf16-nccl", "fsdp", gather_dtype=torch.bfloat16, env=_NCCL),
    Strategy("fsdp-bf16-adamw", "fsdp", gather_dtype=torch.bfloat16, adamw_in_kernel=True),
)}
DEFAULT = "none,ddp,ddp-nccl,ddp-no-overlap,fsdp,fsdp-bf16,fsdp-bf16-nccl,fsdp-bf16-adamw"


@dataclass
class Result:
    strategy: str
    ms_per_step: float
    tokens_per_s: float
    bus_mb: float
    predicted_bus_mb: float
    state_mb: float
    peak_mb: float
    per_collective_mb: dict[str, float] = field(default_factory=dict)
    exposed_pct: float | None = None
    fused_pct: float | None = None
    peer_wait_pct: float | None = None


class _Env:
    """Set environment switches for the duration of a model's construction."""

    def __init__(self, pairs):
        self.pairs, self.old = pairs, {}

    def __enter__(self):
        for k, v in self.pairs:
            self.old[k] = os.environ.get(k)
            os.environ[k] = v

    def __exit__(self, *exc):
        for k, v in self.old.items():
            if v is None:
                os.environ.pop(k, None)
            else:
                os.environ[k] = v
        return False


def make_step(s: Strategy, mesh, config, device, precision, batch, cap_mb) -> tuple[Callable, torch.nn.Module]:
    model = GPT(config, tp_group=mesh.tp_group, device=device)
    adam = dict(lr=1e-4, betas=(0.9, 0.999), eps=1e-8, weight_decay=0.01)
    in_kernel = False
    if mesh.dp_size > 1 and s.kind == "ddp":
        model = DistributedDataParallel(model, process_group=mesh.dp_group, bucket_cap_mb=cap_mb,
                                        overlap_with_backward=s.overlap)
    elif mesh.dp_size > 1 and s.kind == "fsdp":
        kw = {}
        in_kernel = s.adamw_in_kernel and device.type == "cuda" and os.environ.get("MINIDIST_FSDP_FUSED", "1") != "0"
        if in_kernel:
            kw["fused_adamw"] = adam
        model = FullyShardedDataParallel(model, unit_types=(Block,), process_group=mesh.dp_group,
                                         mixed_precision=MixedPrecisionPolicy(param_dtype=s.gather_dtype), **kw)
    opt = None
    if not in_kernel:
        if device.type == "cuda":
            from minidist.optim import FusedAdamW

            opt = FusedAdamW(model.parameters(), **adam)
        else:
            opt = torch.optim.AdamW(model.parameters(), **adam)
    ids, tgt = batch

    def step(_=0):
        if opt is not None:
            opt.zero_grad(set_to_none=True)
        with precision.autocast():
            _, loss = model(ids, tgt)
        loss.backward()
        if opt is not None:
            opt.step()

    return step, model


def _device_seconds(step, iters: int, device) -> float:
    if device.type == "cuda":
        torch.cuda.synchronize()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        for _ in range(iters):
            step()
        b.record()
        b.synchronize()
        sec = a.elapsed_time(b) / 1e3
    else:
        t0 = time.perf_counter()
        for _ in range(iters):
            step()
        sec = time.perf_counter() - t0
    t = torch.tensor([sec], dtype=torch.float64, device=device)
    if dist.is_initialized():
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def run(s: Strategy, args, mesh, config, device, precision) -> Result:
    torch.manual_seed(args.seed)
    g = torch.Generator().manual_seed(args.seed + 10_000 + mesh.dp_rank)
    batch = tuple(torch.randint(0, config.vocab_size, (args.batch_size, config.block_size), generator=g).to(device)
                  for _ in range(2))
    with _Env(s.env if device.type == "cuda" else ()):
        step, model = make_step(s, mesh, config, device, precision, batch, args.bucket_cap_mb)
    for _ in range(args.warmup):
        step()
    if device.type == "cuda":
        torch.cuda.synchronize()
        torch.cuda.reset_peak_memory_stats()
    with record_comm() as stats:
        step()
    sec = _device_seconds(step, args.iters, device)
    local_params = sum(p.numel() for p in (model.module if hasattr(model, "module") else model).parameters())
    if isinstance(model, FullyShardedDataParallel):
        local_params = sum(u.total_numel for u in model._units)
        state = model.memory_summary()["fsdp_state_MB"]
    else:
        state = local_params * 16 / 2**20  # fp32 weights, gradients, Adam m and v
    res = Result(
        strategy=s.name,
        ms_per_step=sec / args.iters * 1e3,
        tokens_per_s=args.batch_size * config.block_size * mesh.dp_size * args.iters / sec,
        bus_mb=stats.total_bus_bytes() / 2**20,
        predicted_bus_mb=s.bus_mb(local_params, mesh.dp_size),
        state_mb=state,
        peak_mb=torch.cuda.max_memory_allocated() / 2**20 if device.type == "cuda" else 0.0,
        per_collective_mb={name: bus / 2**20 for name, _, _, bus in stats.as_rows()},
    )
    if args.trace_dir:
        trace = Path(args.trace_dir) / f"{s.name}_rank{mesh.rank}.json"
        prof = profile_steps(step, num_steps=5, warmup=1, wait=1, trace_path=trace,
                             peer_wait=device.type == "cuda")
        rep = analyze_trace(trace)
        vals = torch.tensor([rep.exposed_fraction_of_step, rep.fused_s / max(rep.wall_s, 1e-12)],
                            dtype=torch.float64, device=device)
        if dist.is_initialized():
            dist.all_reduce(vals, op=dist.ReduceOp.MAX)
        res.exposed_pct, res.fused_pct = float(vals[0]) * 100, float(vals[1]) * 100
        pw = getattr(prof, "md_peer_wait", None)
        if pw is not None and pw.result:
            run_ms = sum(r["run_ms"] for r in pw.result.values())
            res.peer_wait_pct = 100 * sum(r["wait_ms"] for r in pw.result.values()) / max(run_ms, 1e-12)
    return res


def _pct(v) -> str:
    return "-" if v is None else f"{v:.1f}%"


def main(argv=None) -> None:
    p = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    p.add_argument("--strategies", default=DEFAULT, type=lambda v: v.split(","))
    p.add_argument("--tp", type=int, default=1)
    p.add_argument("--layers", type=int, default=8)
    p.add_argument("--heads", type=int, default=8)
    p.add_argument("--embd", type=int, default=512)
    p.add_argument("--vocab", type=int, default=8192)
    p.add_argument("--seq-len", type=int, default=256)
    p.add_argument("--batch-size", type=int, default=8, help="sequences per data-parallel replica")
    p.add_argument("--iters", type=int, default=10)
    p.add_argument("--warmup", type=int, default=3)
    p.add_argument("--bucket-cap-mb", type=float, default=25.0)
    p.add_argument("--seed", type=int, default=1234)
    p.add_argument("--precision", default="fp32", choices=["fp32", "bf16", "auto"])
    p.add_argument("--backend", default=None, choices=[None, "nccl", "gloo"])
    p.add_argument("--trace-dir", default=None, help="profile each strategy; adds the exposed / fused / wait columns")
    p.add_argument("--json", default=None, metavar="PATH", help="rank 0 appends one JSON record per strategy")
    args = p.parse_args(argv)
    unknown = [s for s in args.strategies if s not in STRATEGIES]
    if unknown:
        raise SystemExit(f"unknown strategies {unknown}; choose from {sorted(STRATEGIES)}")

    rank, world, device = init_distributed(backend=args.backend)
    mesh = ParallelMesh(tp_size=args.tp)
    config = GPTConfig(vocab_size=args.vocab, block_size=args.seq_len, n_layer=args.layers, n_head=args.heads,
                       n_embd=args.embd, seed=args.seed)
    precision = resolve_precision(args.precision, device)
    print_rank0(f"\n{mesh.describe()} | {device.type} | {precision} | {config.n_layer}L x {config.n_embd}d, vocab "
                f"{config.vocab_size}, seq {config.block_size}, {args.batch_size} seqs/replica, "
                f"{config.param_count() / 1e6:.1f}M params")
    cols = ["strategy", "ms/step", "tok/s", "bus MB", "model MB", "state MB", "peak MB", "exposed", "fused", "wait"]
    widths = [17, 9, 11, 9, 10, 10, 9, 9, 8, 7]
    print_rank0("".join(f"{c:>{w}}" if i else f"{c:<{w}}" for i, (c, w) in enumerate(zip(cols, widths))))
    results = []
    for name in args.strategies:
        r = run(STRATEGIES[name], args, mesh, config, device, precision)
        results.append(r)
        vals = [r.strategy, f"{r.ms_per_step:.2f}", f"{r.tokens_per_s:.0f}", f"{r.bus_mb:.1f}",
                f"{r.predicted_bus_mb:.1f}", f"{r.state_mb:.1f}", f"{r.peak_mb:.0f}", _pct(r.exposed_pct),
                _pct(r.fused_pct), _pct(r.peer_wait_pct)]
        print_rank0("".join(f"{v:>{w}}" if i else f"{v:<{w}}" for i, (v, w) in enumerate(zip(vals, widths))))
        if args.json and rank == 0:
            with open(args.json, "a") as fh:
                fh.write(json.dumps(dict(asdict(r), world=world, tp=args.tp, precision=args.precision)) + "\n")
    print_rank0("\nbus MB per collective kind (measured, per step and rank):")
    for r in results:
        if r.per_collective_mb:
            print_rank0(f"  {r.strategy:<17}" + ", ".join(f"{k} {v:.1f}" for k, v in sorted(r.per_collective_mb.items())))
    by = {r.strategy: r for r in results}
    pairs = [(a, b) for a, b in (("ddp-nccl", "ddp"), ("ddp-no-overlap", "ddp"), ("fsdp-bf16-nccl", "fsdp-bf16"),
                                 ("fsdp", "fsdp-bf16"), ("fsdp-bf16", "fsdp-bf16-adamw"), ("ddp", "fsdp-bf16"))
             if a in by and b in by]
    if pairs:
        print_rank0("\nspeed-ups (step time of the first / of the second):")
        for a, b in pairs:
            print_rank0(f"  {b:<17} vs {a:<17}{by[a].ms_per_step / by[b].ms_per_step:>7.2f}x")
    shutdown_distributed()


if __name__ == "__main__":
    main()
