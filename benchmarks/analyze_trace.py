#!/usr/bin/env python3
"""Attribute the device time of per-rank Chrome traces (``--profile`` output of the trainer).

    python benchmarks/analyze_trace.py traces/run_rank*.json
    python benchmarks/analyze_trace.py traces/run_rank*.json --kernels 15 --json summary.json

For every trace: timeline, compute, fused compute+collective, library
collectives (hidden / exposed) and idle time (minidist.profiling.analyze_trace).
Across the traces the job-level figure is the *maximum* exposed communication
over ranks -- a collective is only as fast as its slowest participant.
``--kernels N`` lists the N kernels with the most device time in the first
trace with their class, so the fused kernels' share of a step is visible.
``--cpu`` analyses CPU operators even when the trace has kernels.
"""

from __future__ import annotations

import argparse
import csv
import json
import sys
from pathlib import Path

sys.path.insert(0, str(Path(__file__).resolve().parent.parent))

from minidist.profiling import analyze_trace, format_kernel_table, kernel_table  # noqa: E402

_COLUMNS = ("wall_s", "compute_s", "fused_s", "comm_s", "overlapped_s", "exposed_comm_s", "idle_s")


def main(argv=None) -> int:
    p = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    p.add_argument("traces", nargs="+", type=Path)
    p.add_argument("--cpu", action="store_true", help="use CPU operators even if kernels are present")
    p.add_argument("--kernels", type=int, default=0, metavar="N", help="top-N kernel table of the first trace")
    p.add_argument("--csv", type=Path, default=None, help="one row per trace")
    p.add_argument("--json", type=Path, default=None, help="per-trace reports plus the job summary")
    args = p.parse_args(argv)

    reports = {str(t): analyze_trace(t, prefer_device=not args.cpu) for t in args.traces}
    width = max(len(Path(k).name) for k in reports)
    print(f"{'trace':<{width}}" + "".join(f"{c.replace('_s', ''):>14}" for c in _COLUMNS) + "   (ms)")
    for name, r in reports.items():
        d = r.as_dict()
        print(f"{Path(name).name:<{width}}" + "".join(f"{d[c] * 1e3:>14.2f}" for c in _COLUMNS))
    worst_name, worst = max(reports.items(), key=lambda kv: kv[1].exposed_comm_s)
    summary = {
        "traces": len(reports),
        "max_exposed_comm_ms": worst.exposed_comm_s * 1e3,
        "max_exposed_fraction_of_step": max(r.exposed_fraction_of_step for r in reports.values()),
        "worst_trace": worst_name,
        "fused_ms_mean": sum(r.fused_s for r in reports.values()) / len(reports) * 1e3,
    }
    print(f"\njob: exposed library communication {summary['max_exposed_comm_ms']:.2f} ms "
          f"({summary['max_exposed_fraction_of_step'] * 100:.1f}% of the step), max over ranks "
          f"[{Path(worst_name).name}]; fused kernels {summary['fused_ms_mean']:.2f} ms per rank")
    notes = {r.note for r in reports.values() if r.note}
    for n in notes:
        print(f"note: {n}")
    if args.kernels:
        first = args.traces[0]
        print(f"\ntop kernels of {first.name}:")
        print(format_kernel_table(kernel_table(first, top=args.kernels)))
    if args.csv:
        with open(args.csv, "w", newline="") as fh:
            w = csv.writer(fh)
            w.writerow(["trace", "device", *_COLUMNS, "exposed_fraction_of_step"])
            for name, r in reports.items():
                d = r.as_dict()
                w.writerow([name, d["device"], *(f"{d[c]:.6f}" for c in _COLUMNS), f"{d['exposed_fraction_of_step']:.4f}"])
    if args.json:
        args.json.write_text(json.dumps({"summary": summary,
                                         "traces": {k: r.as_dict() for k, r in reports.items()}}, indent=1))
    return 0


if __name__ == "__main__":
    sys.exit(main())
