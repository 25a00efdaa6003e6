#!/usr/bin/env python3
"""Pipeline bubble sweep: measured idle fraction per stage against (P-1)/(M+P-1).

    torchrun --nproc-per-node 4 benchmarks/bench_pipeline.py --microbatches 1,2,4,8,16 --gantt

Runs every schedule for every microbatch count, gathers each stage's report
(wall, busy, comm, measured and theoretical bubble, peak live activations)
with plain collectives, and prints them side by side, optionally with an ASCII
timeline of every stage (reference benchmarks/bench_pipeline.py).  On CUDA the
stage timelines are CUDA-event device time.
"""

from __future__ import annotations

import argparse
import sys
import time
from pathlib import Path

import torch
from torch import nn

sys.path.insert(0, str(Path(__file__).resolve().parent.parent))

from minidist import (  # noqa: E402
    ParallelMesh,
    PipelineStage,
    build_schedule,
    init_distributed,
    partition_layers,
    print_rank0,
    resolve_precision,
    shutdown_distributed,
    theoretical_bubble_fraction,
)
from minidist.comm import all_gather_into_tensor  # noqa: E402
from minidist.models import GPTConfig, build_pipeline_layers  # noqa: E402
from minidist.tensor_parallel import vocab_parallel_cross_entropy  # noqa: E402

KEYS = ("wall_s", "busy_s", "comm_s", "measured_bubble", "theoretical_bubble", "peak_activations_in_flight")
WIDTH = 72


def gather_reports(report: dict, mesh) -> list[dict]:
    local = torch.tensor([float(report[k]) for k in KEYS], dtype=torch.float64, device=mesh.device)
    out = torch.empty(mesh.pp_size * len(KEYS), dtype=torch.float64, device=mesh.device)
    all_gather_into_tensor(out, local, group=mesh.pp_group)
    return [dict(zip(KEYS, row.tolist())) for row in out.view(mesh.pp_size, len(KEYS))]


def gather_ascii(text: str, mesh) -> list[str]:
    enc = text.encode("ascii", "replace")[:WIDTH]
    local = torch.zeros(WIDTH, dtype=torch.uint8, device=mesh.device)
    if enc:
        local[: len(enc)] = torch.frombuffer(bytearray(enc), dtype=torch.uint8)
    out = torch.empty(mesh.pp_size * WIDTH, dtype=torch.uint8, device=mesh.device)
    all_gather_into_tensor(out, local, group=mesh.pp_group)
    return [bytes(r.tolist()).rstrip(b"\0").decode("ascii") for r in out.view(mesh.pp_size, WIDTH)]


def build_stage(config, mesh, device):
    layers = build_pipeline_layers(config, tp_group=mesh.tp_group, device=device)
    mine = partition_layers(layers, mesh.pp_size, mesh.pp_rank)
    start = mesh.tp_rank * (config.vocab_size // mesh.tp_size)

    def loss_fn(logits, targets):
        return vocab_parallel_cross_entropy(logits, targets, group=mesh.tp_group, vocab_start=start)

    return PipelineStage(nn.Sequential(*mine), mesh, loss_fn=loss_fn if mesh.is_last_stage else None)


def main() -> None:
    p = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    p.add_argument("--microbatches", default="1,2,4,8", type=lambda s: [int(x) for x in s.split(",")])
    p.add_argument("--schedules", default="gpipe,1f1b", type=lambda s: s.split(","))
    p.add_argument("--tp", type=int, default=1)
    p.add_argument("--layers", type=int, default=8)
    p.add_argument("--heads", type=int, default=8)
    p.add_argument("--embd", type=int, default=512)
    p.add_argument("--vocab", type=int, default=8192)
    p.add_argument("--seq-len", type=int, default=256)
    p.add_argument("--batch-size", type=int, default=16)
    p.add_argument("--iters", type=int, default=5)
    p.add_argument("--seed", type=int, default=1234)
    p.add_argument("--precision", default="fp32", choices=["fp32", "bf16", "auto"])
    p.add_argument("--backend", default=None, choices=[None, "nccl", "gloo"])
    p.add_argument("--gantt", action="store_true")
    args = p.parse_args()

    rank, world, device = init_distributed(backend=args.backend)
    mesh = ParallelMesh(tp_size=args.tp, pp_size=world // args.tp)
    if mesh.pp_size < 2:
        print_rank0("  pipeline benchmark needs pp_size >= 2; launch more ranks")
        shutdown_distributed()
        return
    config = GPTConfig(vocab_size=args.vocab, block_size=args.seq_len, n_layer=args.layers, n_head=args.heads,
                       n_embd=args.embd, seed=args.seed)
    precision = resolve_precision(args.precision, device)
    g = torch.Generator().manual_seed(args.seed)
    ids = torch.randint(0, config.vocab_size, (args.batch_size, config.block_size), generator=g).to(device)
    tgt = torch.randint(0, config.vocab_size, (args.batch_size, config.block_size), generator=g).to(device)
    print_rank0(f"\n{'=' * 96}\n  pipeline bubble sweep   P={mesh.pp_size} stages   batch={args.batch_size}   "
                f"{config.n_layer}L x {config.n_embd}d   device={device.type}\n{'=' * 96}")
    print_rank0(f"  {'schedule':<10}{'M':>4}{'ms/step':>10}{'measured':>11}{'theory':>9}{'gap':>8}"
                f"{'live acts':>11}{'comm ms':>10}   per-stage busy ms\n  " + "-" * 92)
    for name in args.schedules:
        for m in args.microbatches:
            if args.batch_size % m:
                continue
            stage = build_stage(config, mesh, device)
            opt = torch.optim.SGD(stage.parameters(), lr=0.0)
            sched = build_schedule(name, stage, mesh, m)
            with precision.autocast():
                sched.step(inputs=ids, targets=tgt)
            opt.zero_grad(set_to_none=True)
            if device.type == "cuda":
                torch.cuda.synchronize()
            t0 = time.perf_counter()
            for _ in range(args.iters):
                opt.zero_grad(set_to_none=True)
                with precision.autocast():
                    sched.step(inputs=ids, targets=tgt)
            if device.type == "cuda":
                torch.cuda.synchronize()
            el = (time.perf_counter() - t0) / args.iters
            reps = gather_reports(sched.report(), mesh)
            if mesh.rank == 0:
                meas = max(r["measured_bubble"] for r in reps)
                th = theoretical_bubble_fraction(mesh.pp_size, m)
                live = max(r["peak_activations_in_flight"] for r in reps)
                comm_ms = max(r["comm_s"] for r in reps) * 1e3
                busy = "  ".join(f"{r['busy_s'] * 1e3:.1f}" for r in reps)
                print_rank0(f"  {name:<10}{m:>4}{el * 1e3:>10.2f}{meas * 100:>10.1f}%{th * 100:>8.1f}%"
                            f"{(meas - th) * 100:>+7.1f}%{live:>11.0f}{comm_ms:>10.2f}   {busy}")
            if args.gantt and m == args.microbatches[-1]:
                rows = gather_ascii(sched.timeline.ascii_gantt(WIDTH), mesh)
                if mesh.rank == 0:
                    print_rank0(f"\n  {name} timeline, M={m} (F=forward B=backward >=send <=recv .=idle)")
                    for i, r in enumerate(rows):
                        print_rank0(f"    stage {i}  {r}")
                    print_rank0("")
            del stage, sched, opt
    shutdown_distributed()


if __name__ == "__main__":
    main()
