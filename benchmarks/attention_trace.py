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
    p.add_argument("--bwd", action="store_true", help="trace the backward kernel instead (head_dim 64)")
    a = p.parse_args(argv)
    import torch

    from minidist.ops import _native as nat
    from minidist.ops import kernels as K

    B, H, S, D = (int(v) for v in a.shape.split(","))
    qkv = torch.randn(B * S, 3 * H * D, device="cuda").bfloat16()
    for _ in range(3):
        K.attention_fwd(qkv, B, S, H, D, impl="tc")
    torch.cuda.synchronize()
    if a.bwd:
        return _bwd(K, nat, qkv, B, H, S, D, a)
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


def _bwd(K, nat, qkv, B, H, S, D, a) -> int:
    """Backward trace (head_dim 64 kernel).  Compute-warp slots: 1 scores ready, 2 first
    half of P / dS computed, 3 P / dS buffers free, 4 next block's lse / delta staged, 10
    first half stored, 13 / 14 second half's score load issued / complete, 15 second half
    computed, 16.. P / dS handed to the MMA warp (per warp); MMA slots 12 scores issued, 5 P / dS received, 7 dQ TMEM free, 8 dV issued;
    9 dQ drained; 11 Q / dO load issued."""
    import torch

    y, lse = K.attention_fwd(qkv, B, S, H, D, impl="tc")
    dy = torch.randn_like(y)
    for _ in range(3):
        K.attention_bwd(qkv, y, dy, lse, B, S, H, D, impl="tc")
    torch.cuda.synchronize()
    tr = K.attention_pipeline_trace(lambda: K.attention_bwd(qkv, y, dy, lse, B, S, H, D, impl="tc")).tolist()
    nat.check_status()
    med = lambda xs: statistics.median(xs) if xs else float("nan")  # noqa: E731
    rows = [(g, r) for g, r in enumerate(tr) if r[1] and r[16]][a.skip:]
    out = {"shape": [B, H, S, D], "blocks": len(rows)}
    out["scores ready -> first half computed"] = med([r[2] - r[1] for _, r in rows if r[2]])
    out["first half -> buffers free"] = med([r[3] - r[2] for _, r in rows if r[3] and r[2]])
    out["buffers free -> next lse / delta staged"] = med([r[4] - r[3] for _, r in rows if r[4] and r[3]])
    out["-> first half P^T / dS^T stored"] = med([r[10] - r[4] for _, r in rows if r[10] and r[4]])
    out["-> second half scores loaded"] = med([r[14] - r[10] for _, r in rows if r[14] and r[10]])
    out["-> second half computed"] = med([r[15] - r[14] for _, r in rows if r[15] and r[14]])
    out["-> P / dS handed (warp 2)"] = med([r[16] - r[15] for _, r in rows if r[15]])
    out["buffers free -> P / dS handed (warp 2)"] = med([r[16] - r[3] for _, r in rows if r[3]])
    periods = [tr[g + 1][1] - tr[g][1] for g in range(a.skip, 63) if tr[g][1] and tr[g + 1][1]]
    out["block period (median)"] = med(periods)
    out["block period (max)"] = max(periods) if periods else float("nan")
    out["scores issue -> scores ready"] = med([r[1] - r[12] for _, r in rows if r[12]])
    for k, v in out.items():
        print(f"{k:>52}: {v}")
    print("\nper block (cycles from block 0's scores-ready): scores issued, ready, handed, dV issued, dQ drained")
    base = tr[0][1]
    for g in range(min(40, len(tr))):
        r = tr[g]
        if not r[1]:
            break
        print(g, *[(r[i] - base) if r[i] else -1 for i in (12, 1, 16, 8, 9)])
    if a.json:
        Path(a.json).write_text(json.dumps({"raw": tr, "summary": out}, indent=1))
    return 0


if __name__ == "__main__":
    sys.exit(main())
