#!/usr/bin/env python3
"""Where one training step of a benchmark configuration spends its device time.

    python benchmarks/profile_step.py --config gpt1.5b-fsdp
    torchrun --nproc-per-node 8 benchmarks/profile_step.py --gpus 8 --config gpt2s-ddp --trace-dir traces

Builds the configuration exactly as ``bench.py`` does (our arm), runs a few
warm-up steps, then profiles ``--steps`` eager steps with torch.profiler and
prints, on rank 0: the kernels with the most device time per step and their
class (fused compute+collective / library collective / compute), the step's
time by class with exposed communication (max over ranks), and -- on more
than one GPU -- the fused kernels' device-side peer-wait share.  With
``--trace-dir`` every rank's Chrome trace is kept for benchmarks/analyze_trace.py.
"""

from __future__ import annotations

import argparse
import json
import os
import sys
import tempfile
from pathlib import Path

ROOT = Path(__file__).resolve().parent.parent
sys.path.insert(0, str(ROOT))

import bench  # noqa: E402


def main(argv=None) -> int:
    p = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    p.add_argument("--config", choices=sorted(bench.CONFIGS), default="gpt2s-ddp")
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=3)
    p.add_argument("--warmup", type=int, default=3)
    p.add_argument("--top", type=int, default=25)
    p.add_argument("--schedule", choices=["1f1b", "gpipe"], default="1f1b")
    p.add_argument("--trace-dir", default=None)
    p.add_argument("--json", default=None, metavar="PATH", help="rank 0 writes the tables as JSON")
    args = p.parse_args(argv)

    import torch
    import torch.distributed as dist

    from minidist.profiling import analyze_trace, format_kernel_table, kernel_table, profile_steps

    world = int(os.environ.get("WORLD_SIZE", "1"))
    c = bench.resolve_config(args.config, world)
    ns = argparse.Namespace(gpus=args.gpus, device="cuda")
    rank, world, _ = bench.setup(ns)
    built = bench.build("ours", c, world, 1234, graph=False, device="cuda", schedule=args.schedule)
    batches = bench.make_batches(args.warmup + 1, c, built.dp_rank, 1234, pinned=False)
    for i in range(args.warmup):
        built.step(*batches[i])
    torch.cuda.synchronize()
    tdir = Path(args.trace_dir or tempfile.mkdtemp(prefix="md_prof_"))
    trace = tdir / f"{args.config}_rank{rank}.json"
    prof = profile_steps(lambda _: built.step(*batches[-1]), num_steps=args.steps + 2, warmup=1, wait=1,
                         trace_path=trace, record_shapes=False, peer_wait=world > 1)
    rows = kernel_table(trace, top=args.top)
    rep = analyze_trace(trace)
    exposed = torch.tensor([rep.exposed_comm_s], dtype=torch.float64, device="cuda")
    if world > 1:
        dist.all_reduce(exposed, op=dist.ReduceOp.MAX)
    if rank == 0:
        per_step = args.steps
        print(f"\n{args.config} on {world} GPU(s), {per_step} profiled steps "
              f"(times below are per step; the profiler adds overhead, not a benchmark number)")
        for r in rows:
            r.device_time_us /= per_step
            r.count = r.count // per_step
        print(format_kernel_table(rows))
        print(f"\ntimeline by class (rank 0, per step):")
        for k in ("wall_s", "compute_s", "fused_s", "comm_s", "exposed_comm_s", "idle_s"):
            print(f"  {k[:-2]:<14}{getattr(rep, k) / per_step * 1e3:>9.2f} ms")
        print(f"  exposed comm, max over ranks: {float(exposed) / per_step * 1e3:.2f} ms per step")
        pw = getattr(prof, "md_peer_wait", None)
        if pw is not None and pw.result:
            print("\npeer-wait counters (summed over CTAs, all profiled steps):")
            print(pw.format())
        if args.json:
            Path(args.json).write_text(json.dumps({
                "config": args.config, "world": world, "steps": per_step,
                "kernels": [r.__dict__ for r in rows], "overlap": rep.as_dict(),
                "exposed_comm_ms_max": float(exposed) / per_step * 1e3,
                "peer_wait": pw.result if pw is not None else None}, indent=1))
    if world > 1:
        from minidist.parallel import symm

        symm.release_all()
        dist.barrier()
        dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())
