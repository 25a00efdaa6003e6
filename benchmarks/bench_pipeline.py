#!/usr/bin/env python3
"""Pipeline schedules under a microbatch sweep: step time, bubble against (P-1)/(M+P-1), live activations.

    torchrun --nproc-per-node 4 benchmarks/bench_pipeline.py --microbatches 1,2,4,8,16 --gantt
    torchrun --nproc-per-node 8 benchmarks/bench_pipeline.py --tp 2 --precision bf16 --layers 16 --embd 1024

For every (schedule, M) the stage runs ``--iters`` steps, timed on the device
(CUDA events; the maximum over ranks), then each rank contributes one record
-- its stage timeline's busy / comm / bubble figures, its peak live
activations and (CUDA) its peak memory -- through ``all_gather_object`` over
the pipeline group.  Rank 0 prints one line per (schedule, M) with the worst
stage's bubble beside the theoretical fraction, and with ``--gantt`` one chart
of the last step in which every stage is drawn on the same time axis (the
stage clocks start together after a barrier), so fill and drain show as
staircases.  Optimizer: SGD with lr 0, so each step sees the same weights.
With ``--precision bf16`` on CUDA the blocks run the fused kernels and the
last stage's LM head computes its loss fused (``LMHead.loss_only``).
"""

from __future__ import annotations

import argparse
import json
import sys
from pathlib import Path

import torch
import torch.distributed as dist
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
from minidist.models import GPTConfig, LMHead, build_pipeline_layers  # noqa: E402
from minidist.tensor_parallel import vocab_parallel_cross_entropy  # noqa: E402

_GLYPH = {"forward": "F", "backward": "B", "send": ">", "recv": "<"}


def stage_for(config, mesh, device, fused: bool) -> PipelineStage:
    mine = partition_layers(build_pipeline_layers(config, tp_group=mesh.tp_group, device=device),
                            mesh.pp_size, mesh.pp_rank)
    loss_fn = None
    if mesh.is_last_stage:
        head = mine[-1]
        if fused and isinstance(head, LMHead):
            head.loss_only = True
            loss_fn = head.loss
        else:
            start = mesh.tp_rank * (config.vocab_size // mesh.tp_size)

            def loss_fn(logits, targets):
                return vocab_parallel_cross_entropy(logits, targets, group=mesh.tp_group, vocab_start=start)
    return PipelineStage(nn.Sequential(*mine), mesh, loss_fn=loss_fn)


def chart(per_stage: list[list[tuple[str, int, float, float]]], width: int) -> list[str]:
    """One row per stage on a shared time axis (F/B compute, >/< send/recv, . idle)."""
    end = max((e for evs in per_stage for _, _, _, e in evs), default=0.0)
    rows = []
    for evs in per_stage:
        row = ["."] * width
        for kind, _, b, e in sorted(evs, key=lambda ev: ev[0] not in ("forward", "backward")):
            lo = int(b / end * (width - 1)) if end else 0
            hi = max(lo, int(e / end * (width - 1)) if end else 0)
            for i in range(lo, min(hi + 1, width)):
                if row[i] == "." or kind in ("forward", "backward"):
                    row[i] = _GLYPH.get(kind, "?")
        rows.append("".join(row))
    return rows


def main(argv=None) -> None:
    p = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    p.add_argument("--microbatches", default="1,2,4,8", type=lambda v: [int(x) for x in v.split(",")])
    p.add_argument("--schedules", default="gpipe,1f1b", type=lambda v: v.split(","))
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
    p.add_argument("--width", type=int, default=80)
    p.add_argument("--json", default=None, metavar="PATH", help="rank 0 appends one JSON record per (schedule, M)")
    args = p.parse_args(argv)

    rank, world, device = init_distributed(backend=args.backend)
    mesh = ParallelMesh(tp_size=args.tp, pp_size=world // args.tp)
    if mesh.pp_size < 2:
        print_rank0("pipeline benchmark needs at least two stages (world / tp >= 2)")
        shutdown_distributed()
        return
    config = GPTConfig(vocab_size=args.vocab, block_size=args.seq_len, n_layer=args.layers, n_head=args.heads,
                       n_embd=args.embd, seed=args.seed)
    precision = resolve_precision(args.precision, device)
    fused = device.type == "cuda" and precision.enabled and precision.dtype == torch.bfloat16
    g = torch.Generator().manual_seed(args.seed)
    ids, tgt = (torch.randint(0, config.vocab_size, (args.batch_size, config.block_size), generator=g).to(device)
                for _ in range(2))
    cuda = device.type == "cuda"
    print_rank0(f"\nP = {mesh.pp_size} stages x tp {mesh.tp_size} | {config.n_layer}L x {config.n_embd}d | "
                f"batch {args.batch_size} x {config.block_size} | {device.type} {precision}")
    print_rank0(f"{'schedule':<9}{'M':>4}{'ms/step':>10}{'bubble':>9}{'theory':>9}{'excess':>9}{'live acts':>11}"
                f"{'comm ms':>9}{'peak GB':>9}   busy ms per stage")
    for name in args.schedules:
        for m in args.microbatches:
            if args.batch_size % m:
                print_rank0(f"{name:<9}{m:>4}   skipped: batch {args.batch_size} not divisible")
                continue
            stage = stage_for(config, mesh, device, fused)
            opt = torch.optim.SGD(stage.parameters(), lr=0.0)
            sched = build_schedule(name, stage, mesh, m)

            def step():
                opt.zero_grad(set_to_none=True)
                with precision.autocast():
                    sched.step(inputs=ids, targets=tgt)
                opt.step()

            step()  # headers, communicators, lazy kernel set-up
            if cuda:
                torch.cuda.synchronize()
                torch.cuda.reset_peak_memory_stats()
            dist.barrier()
            if cuda:
                a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                a.record()
            else:
                import time

                t0 = time.perf_counter()
            for _ in range(args.iters):
                step()
            if cuda:
                b.record()
                b.synchronize()
                sec = a.elapsed_time(b) / 1e3
            else:
                sec = time.perf_counter() - t0
            t = torch.tensor([sec / args.iters], dtype=torch.float64, device=device)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            rep = sched.report()
            rec = dict(rep, stage=mesh.pp_rank, events=list(sched.timeline.events) if args.gantt else [],
                       peak_gb=torch.cuda.max_memory_allocated() / 2**30 if cuda else 0.0)
            recs = [None] * mesh.pp_size
            dist.all_gather_object(recs, rec, group=mesh.pp_group)
            if rank == 0:
                recs.sort(key=lambda r: r["stage"])
                worst = max(r["measured_bubble"] for r in recs)
                theory = theoretical_bubble_fraction(mesh.pp_size, m)
                live = max(r["peak_activations_in_flight"] for r in recs)
                comm_ms = max(r["comm_s"] for r in recs) * 1e3
                peak = max(r["peak_gb"] for r in recs)
                busy = " ".join(f"{r['busy_s'] * 1e3:.1f}" for r in recs)
                print_rank0(f"{name:<9}{m:>4}{float(t) * 1e3:>10.2f}{worst * 100:>8.1f}%{theory * 100:>8.1f}%"
                            f"{(worst - theory) * 100:>+8.1f}%{live:>11.0f}{comm_ms:>9.2f}{peak:>9.2f}   {busy}")
                if args.json:
                    with open(args.json, "a") as fh:
                        fh.write(json.dumps(dict(schedule=name, microbatches=m, ms_per_step=float(t) * 1e3,
                                                 bubble=worst, theoretical_bubble=theory, live_activations=live,
                                                 stages=[{k: v for k, v in r.items() if k != "events"}
                                                         for r in recs])) + "\n")
                if args.gantt and m == args.microbatches[-1]:
                    print_rank0(f"  {name}, M={m}, last step (F forward, B backward, > send, < recv, . idle):")
                    for i, row in enumerate(chart([r["events"] for r in recs], args.width)):
                        print_rank0(f"  stage {i} |{row}|")
            del stage, sched, opt
    shutdown_distributed()


if __name__ == "__main__":
    main()
