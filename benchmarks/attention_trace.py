#!/usr/bin/env python3
"""Where one 128 x 128 key block of the tcgen05 attention forward spends its cycles.

    python benchmarks/attention_trace.py --shape 16,12,1024,64
    python benchmarks/attention_trace.py --shape 4,16,2048,128 --json trace.json

Runs the forward a few times, then once with the kernel's pipeline trace on: CTA 0 stamps
``clock64()`` at each hand-off of its first 64 key blocks (TMA issue of K / V, MMA issue of
S = QK^T and O += PV, and in the softmax warps: scores ready, scores loaded, row max done,
exponentials done with P written to TMEM, O synchronised, P handed to the MMA warp).  Prints, over the steady-state blocks (the first
``--skip`` are dropped), the median cycles of each softmax stage and of the block period,
and how long the MMA warp waits for P.  Analysis only; timing numbers come from
kernel_bench.py.
"""

from __future__ import annotations

import argparse
import json
import statistics
import sys
from pathlib import Path

sys.path.insert(0, str(Path(__file__).resolve().parent.parent))

STAGES = [("scores ready -> loaded", 0, 1), ("loaded -> row max", 1, 2), ("row max -> exps, P in TMEM", 2, 3),
          ("-> O synchronised / rescaled", 3, 4), ("-> P handed to MMA", 4, 5)]


def main(argv=None) -> int:
    p = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    p.add_argument("--shape", default="16,12,1024,64", help="B,H,S,D")
    p.add_argument("--skip", type=int, default=2)
    p.add_argument("--json", default=None)
    a = p.parse_args(argv)
    import torch

    from minidist.ops import _native as nat
    from minidist.ops import kernels as K

    B, H, S, D = (int(v) for v in a.shape.split(","))
    qkv = torch.randn(B * S, 3 * H * D, device="cuda").bfloat16()
    for _ in range(3):
        K.attention_fwd(qkv, B, S, H, D, impl="tc")
    torch.cuda.synchronize()
    tr = K.attention_pipeline_trace(lambda: K.attention_fwd(qkv, B, S, H, D, impl="tc")).tolist()
    nat.check_status()
    rows = [r for r in tr if r[0] and r[5]][a.skip:]
    out = {"shape": [B, H, S, D], "blocks": len(rows)}
    med = lambda xs: statistics.median(xs) if xs else float("nan")  # noqa: E731
    for name, i, j in STAGES:
        for w, off in (("warp 2", 0), ("warp 6", 6)):
            xs = [r[off + j] - r[off + i] for r in rows if r[off + i] and r[off + j]]
            if xs:
                out[f"{w}: {name}"] = med(xs)
    periods = [tr[g + 1][0] - tr[g][0] for g in range(a.skip, 63) if tr[g][0] and tr[g + 1][0]]
    out["block period (scores ready to next scores ready)"] = med(periods)
    out["P handed over -> MMA issues PV"] = med([r[13] - r[5] for r in rows if r[13] and r[5]])
    out["S issue -> scores ready"] = med([r[0] - r[12] for r in rows if r[0] and r[12]])
    for k, v in out.items():
        print(f"{k:>52}: {v}")
    if a.json:
        Path(a.json).write_text(json.dumps({"raw": tr, "summary": out}, indent=1))
    return 0


if __name__ == "__main__":
    sys.exit(main())
