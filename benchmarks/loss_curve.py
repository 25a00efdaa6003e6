#!/usr/bin/env python3
"""Training-loss curve of one arm on a benchmark configuration, and the comparison of two curves.

    python benchmarks/loss_curve.py --impl ours --steps 300 --out ours.json
    python benchmarks/loss_curve.py --impl reference --steps 300 --out ref.json
    python benchmarks/loss_curve.py --compare ours.json ref.json

Both arms are built exactly as in ``bench.py`` (same seeds: bit-identical
initial weights, the same token batches ``seed + step*10000 + dp_rank``, AdamW
lr 3e-4, bf16 autocast), and every step's loss is read back.  The comparison
prints the largest absolute loss difference over the steps, the mean
difference over the last 50, and both final losses.  The tokens are uniform
random, so the loss falls from ln(vocab) toward the entropy of the
distribution; what matters here is that the two curves track each other.
"""

from __future__ import annotations

import argparse
import json
import os
import sys
from pathlib import Path

ROOT = Path(__file__).resolve().parent.parent
sys.path.insert(0, str(ROOT))


def run(args) -> int:
    import bench

    world = int(os.environ.get("WORLD_SIZE", "1"))
    c = bench.resolve_config(args.config, world)
    rank, world, _ = bench.setup(argparse.Namespace(gpus=world, device=args.device))
    # Eager steps on both arms, so both see batches 0, 1, 2, ... in order (a CUDA-graph
    # capture would spend its warm-up steps on one fixed batch).
    built = bench.build(args.impl, c, world, args.seed, graph=False, device=args.device)
    batches = bench.make_batches(args.steps, c, built.dp_rank, args.seed, pinned=False, device=args.device)
    losses = [bench._loss_value(built.step(ids, tgt), built, args.device) for ids, tgt in batches]
    if rank == 0:
        Path(args.out).write_text(json.dumps({"impl": args.impl, "config": args.config, "world": world,
                                              "losses": losses}))
        print(f"{args.impl}: {len(losses)} steps, loss {losses[0]:.4f} -> {losses[-1]:.4f}")
    if world > 1:
        import torch.distributed as dist

        if args.impl == "ours" and args.device == "cuda":
            from minidist.parallel import symm

            symm.release_all()
        dist.barrier()
        dist.destroy_process_group()
    return 0


def compare(a_path: str, b_path: str) -> int:
    a = json.loads(Path(a_path).read_text())
    b = json.loads(Path(b_path).read_text())
    pairs = list(zip(a["losses"], b["losses"]))
    diffs = [abs(x - y) for x, y in pairs]
    tail = diffs[-50:]
    out = {"steps_compared": len(pairs), "max_abs_diff": max(diffs), "mean_abs_diff_last50": sum(tail) / len(tail),
           f"final_{a['impl']}": pairs[-1][0], f"final_{b['impl']}": pairs[-1][1]}
    print(json.dumps(out))
    return 0


def main(argv=None) -> int:
    p = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    p.add_argument("--impl", choices=["ours", "reference"], default="ours")
    p.add_argument("--config", default="gpt2s-ddp")
    p.add_argument("--steps", type=int, default=300)
    p.add_argument("--seed", type=int, default=1234)
    p.add_argument("--device", choices=["cuda", "cpu"], default="cuda")
    p.add_argument("--out", default="loss_curve.json")
    p.add_argument("--compare", nargs=2, metavar=("A", "B"))
    args = p.parse_args(argv)
    if args.compare:
        return compare(*args.compare)
    return run(args)


if __name__ == "__main__":
    sys.exit(main())
