#!/usr/bin/env python3
"""Overlap report from one or more Chrome traces (``--profile`` of examples/train_gpt.py,
``--profile-dir`` of bench_parallelism.py).

    python benchmarks/analyze_trace.py traces/trace_ddp_rank0.json --csv overlap.csv
"""

from __future__ import annotations

import argparse
import csv
import sys
from pathlib import Path

sys.path.insert(0, str(Path(__file__).resolve().parent.parent))

from minidist.profiling import analyze_trace  # noqa: E402


def main() -> None:
    p = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    p.add_argument("traces", nargs="+", type=Path)
    p.add_argument("--csv", type=Path, default=None)
    p.add_argument("--cpu", action="store_true", help="force the CPU-operator view")
    args = p.parse_args()
    rows = []
    for path in args.traces:
        if not path.exists():
            print(f"  {path}: not found", file=sys.stderr)
            continue
        r = analyze_trace(path, prefer_device=not args.cpu)
        print(f"\n{path.name}\n{r.format()}")
        rows.append((path.name, r))
    if args.csv and rows:
        with open(args.csv, "w", newline="") as fh:
            w = csv.writer(fh)
            w.writerow(["trace", "device", "wall_s", "compute_s", "comm_s", "overlapped_s", "fused_s",
                        "exposed_comm_s", "overlap_fraction", "exposed_fraction_of_step"])
            for name, r in rows:
                w.writerow([name, r.device, f"{r.wall_s:.6f}", f"{r.compute_s:.6f}", f"{r.comm_s:.6f}",
                            f"{r.overlapped_s:.6f}", f"{r.fused_s:.6f}", f"{r.exposed_comm_s:.6f}",
                            f"{r.overlap_fraction:.4f}", f"{r.exposed_fraction_of_step:.4f}"])
        print(f"\nwrote {args.csv}")


if __name__ == "__main__":
    main()
