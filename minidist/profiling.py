"""Profiler integration: per-collective breakdowns and communication/compute overlap.

:func:`profile_steps` runs a step function under ``torch.profiler`` with a
wait/warm-up/active schedule and exports a Chrome trace.
:func:`summarize_collectives` groups the event table by collective kind, and
:func:`analyze_trace` measures how much communication ran with no compute
beside it, by interval arithmetic over the trace's kernels (reference
profiling.py:1-38, 295-361): merge the intervals of each category, intersect,
and report ``exposed = |comm| - |comm & compute|``.

B200 additions.  The fused kernels of :mod:`minidist.parallel` carry stable
name prefixes (``md_ar_``, ``md_rs_``, ``md_ag_``, ``md_gemm_rs``,
``md_gemm_ar``, ``md_ag_gemm``).  They are classified with their collective
kind *and* counted as fused: a fused kernel overlaps its own communication
with its own math, so it is reported in ``fused_s`` rather than as exposed
communication.  NCCL kernels and ``c10d::`` operators are classified as in the
reference.  On a Gloo/CPU trace there are no kernels; the analysis falls back
to CPU operators and says so.
"""

from __future__ import annotations

import gzip
import json
from collections.abc import Callable, Iterable, Sequence
from dataclasses import dataclass, field
from pathlib import Path

import torch
from torch.profiler import ProfilerActivity, profile, schedule

__all__ = [
    "COLLECTIVE_PATTERNS",
    "FUSED_PATTERNS",
    "OverlapReport",
    "CollectiveRow",
    "profile_steps",
    "summarize_collectives",
    "analyze_trace",
    "format_collective_table",
]

COLLECTIVE_PATTERNS: tuple[str, ...] = (
    "nccl",
    "c10d::",
    "record_param_comms",
    "ProcessGroupNCCL",
    "ProcessGroupGloo",
)

# Fused compute+collective kernels of this framework: name fragment -> kind.
FUSED_PATTERNS: dict[str, str] = {
    "md_gemm_ar": "all_reduce",
    "md_gemm_rs": "reduce_scatter",
    "md_ag_gemm": "all_gather",
    "md_ar_": "all_reduce",
    "md_rs_": "reduce_scatter",
    "md_ag_": "all_gather",
    "md_ce_tp": "all_reduce",  # the vocab-parallel cross-entropy statistics exchange
}

_KINDS = {
    "all_reduce": ("allreduce", "all_reduce"),
    "all_gather": ("allgather", "all_gather", "_allgather_base"),
    "reduce_scatter": ("reducescatter", "reduce_scatter"),
    "broadcast": ("broadcast",),
    "send_recv": ("send", "recv", "sendrecv", "p2p"),
    "barrier": ("barrier",),
}


def _classify(name: str) -> str | None:
    low = name.lower()
    for frag, kind in FUSED_PATTERNS.items():
        if frag in low:
            return kind
    for kind, needles in _KINDS.items():
        if any(n in low for n in needles):
            return kind
    return None


def _is_fused(name: str) -> bool:
    low = name.lower()
    return any(frag in low for frag in FUSED_PATTERNS)


def _is_collective(name: str) -> bool:
    low = name.lower()
    return any(p.lower() in low for p in COLLECTIVE_PATTERNS) or _is_fused(name)


# ---------------------------------------------------------------------------
# Running the profiler
# ---------------------------------------------------------------------------


def profile_steps(
    step_fn: Callable[[int], None],
    num_steps: int = 6,
    warmup: int = 2,
    wait: int = 1,
    trace_path: str | Path | None = None,
    record_shapes: bool = True,
    with_stack: bool = False,
    activities: Sequence[ProfilerActivity] | None = None,
):
    """Run ``step_fn(step)`` ``num_steps`` times under the profiler; optionally export a Chrome trace.

    The first ``wait`` steps are ignored and the next ``warmup`` traced but
    discarded, so one-off costs (communicator creation, allocator growth)
    stay out of the active window.
    """
    if activities is None:
        activities = [ProfilerActivity.CPU]
        if torch.cuda.is_available():
            activities.append(ProfilerActivity.CUDA)
    active = max(1, num_steps - wait - warmup)
    with profile(activities=list(activities),
                 schedule=schedule(wait=wait, warmup=warmup, active=active, repeat=1),
                 record_shapes=record_shapes, with_stack=with_stack, profile_memory=True) as prof:
        for step in range(num_steps):
            step_fn(step)
            prof.step()
    if trace_path is not None:
        trace_path = Path(trace_path)
        trace_path.parent.mkdir(parents=True, exist_ok=True)
        prof.export_chrome_trace(str(trace_path))
    return prof


# ---------------------------------------------------------------------------
# Event-table summary
# ---------------------------------------------------------------------------


@dataclass
class CollectiveRow:
    kind: str
    count: int
    self_time_us: float
    device_time_us: float
    fused: bool = False

    @property
    def avg_us(self) -> float:
        return self.self_time_us / max(1, self.count)


def summarize_collectives(prof) -> list[CollectiveRow]:
    """Per-kind totals of collective events (fused kernels get their own ``<kind>+fused`` rows)."""
    rows: dict[str, CollectiveRow] = {}
    for evt in prof.key_averages():
        if not _is_collective(evt.key):
            continue
        fused = _is_fused(evt.key)
        kind = (_classify(evt.key) or "other") + ("+fused" if fused else "")
        row = rows.setdefault(kind, CollectiveRow(kind, 0, 0.0, 0.0, fused))
        row.count += evt.count
        row.self_time_us += float(getattr(evt, "self_cpu_time_total", 0.0) or 0.0)
        dev = 0.0
        for attr in ("self_device_time_total", "self_cuda_time_total"):
            dev = float(getattr(evt, attr, 0.0) or 0.0)
            if dev:
                break
        row.device_time_us += dev
    return sorted(rows.values(), key=lambda r: -max(r.device_time_us, r.self_time_us))


def format_collective_table(rows: Iterable[CollectiveRow]) -> str:
    rows = list(rows)
    if not rows:
        return "  (no collective events recorded)"
    out = [f"  {'collective':<22}{'count':>8}{'device ms':>12}{'cpu ms':>10}{'avg us':>10}", "  " + "-" * 62]
    for r in rows:
        out.append(f"  {r.kind:<22}{r.count:>8}{r.device_time_us / 1e3:>12.2f}"
                   f"{r.self_time_us / 1e3:>10.2f}{r.avg_us:>10.1f}")
    return "\n".join(out)


# ---------------------------------------------------------------------------
# Interval arithmetic
# ---------------------------------------------------------------------------

Interval = tuple[float, float]


def _merge(intervals: list[Interval]) -> list[Interval]:
    """Union of intervals as a sorted, disjoint list (touching intervals join)."""
    out: list[Interval] = []
    for b, e in sorted(intervals):
        if out and b <= out[-1][1]:
            if e > out[-1][1]:
                out[-1] = (out[-1][0], e)
        else:
            out.append((b, e))
    return out


def _total(intervals: Iterable[Interval]) -> float:
    return sum(e - b for b, e in intervals)


def _intersect(a: list[Interval], b: list[Interval]) -> list[Interval]:
    """Intersection of two merged lists (linear sweep)."""
    out: list[Interval] = []
    i = j = 0
    while i < len(a) and j < len(b):
        lo, hi = max(a[i][0], b[j][0]), min(a[i][1], b[j][1])
        if lo < hi:
            out.append((lo, hi))
        if a[i][1] < b[j][1]:
            i += 1
        else:
            j += 1
    return out


def _subtract(a: list[Interval], b: list[Interval]) -> list[Interval]:
    """``a`` minus ``b`` for merged lists."""
    out: list[Interval] = []
    j = 0
    for lo, hi in a:
        while j < len(b) and b[j][1] <= lo:
            j += 1
        cur = lo
        k = j
        while k < len(b) and b[k][0] < hi:
            if b[k][0] > cur:
                out.append((cur, b[k][0]))
            cur = max(cur, b[k][1])
            k += 1
        if cur < hi:
            out.append((cur, hi))
    return out


@dataclass
class OverlapReport:
    """Communication/compute overlap of one trace, in seconds."""

    device: str
    wall_s: float = 0.0
    compute_s: float = 0.0
    comm_s: float = 0.0
    overlapped_s: float = 0.0
    fused_s: float = 0.0
    num_comm_events: int = 0
    num_compute_events: int = 0
    per_kind_s: dict[str, float] = field(default_factory=dict)
    note: str = ""

    @property
    def exposed_comm_s(self) -> float:
        return max(0.0, self.comm_s - self.overlapped_s)

    @property
    def overlap_fraction(self) -> float:
        return self.overlapped_s / self.comm_s if self.comm_s > 0 else 0.0

    @property
    def exposed_fraction_of_step(self) -> float:
        return self.exposed_comm_s / self.wall_s if self.wall_s > 0 else 0.0

    def format(self) -> str:
        lines = [
            f"  device            : {self.device}",
            f"  wall              : {self.wall_s * 1e3:.2f} ms",
            f"  compute (busy)    : {self.compute_s * 1e3:.2f} ms ({self.num_compute_events} events)",
            f"  communication     : {self.comm_s * 1e3:.2f} ms ({self.num_comm_events} events)",
            f"  overlapped        : {self.overlapped_s * 1e3:.2f} ms ({self.overlap_fraction * 100:.1f}% of comm hidden)",
            f"  exposed comm      : {self.exposed_comm_s * 1e3:.2f} ms ({self.exposed_fraction_of_step * 100:.1f}% of step)",
        ]
        if self.fused_s > 0:
            lines.append(f"  fused comm+compute: {self.fused_s * 1e3:.2f} ms (kernels that overlap internally)")
        if self.per_kind_s:
            lines.append("  by collective     :")
            for kind, sec in sorted(self.per_kind_s.items(), key=lambda kv: -kv[1]):
                lines.append(f"      {kind:<22}{sec * 1e3:>10.2f} ms")
        if self.note:
            lines.append(f"  note              : {self.note}")
        return "\n".join(lines)


def _load_trace(path: str | Path) -> dict:
    path = Path(path)
    opener = gzip.open if path.suffix == ".gz" else open
    with opener(path, "rt") as fh:
        return json.load(fh)


def analyze_trace(path: str | Path, prefer_device: bool = True) -> OverlapReport:
    """Overlap report from a Chrome trace (GPU kernels if present, else CPU operators)."""
    events = [e for e in _load_trace(path).get("traceEvents", []) if e.get("ph") == "X"]
    use_device = prefer_device and any(e.get("cat") == "kernel" for e in events)
    if use_device:
        pool = [e for e in events if e.get("cat") == "kernel"]
        device, note = "cuda", ""
    else:
        pool = [e for e in events if e.get("cat") in ("cpu_op", "user_annotation")]
        device = "cpu"
        note = ("Gloo/CPU trace: collectives are blocking CPU operators, so overlap is structurally ~0 here. "
                "Run on CUDA+NCCL for a meaningful number.")

    comm_iv: list[Interval] = []
    comp_iv: list[Interval] = []
    fused_iv: list[Interval] = []
    per_kind: dict[str, list[Interval]] = {}
    n_comm = n_comp = 0
    for e in pool:
        b = float(e["ts"]) * 1e-6
        iv = (b, b + float(e.get("dur", 0)) * 1e-6)
        name = e.get("name", "")
        if _is_fused(name):
            fused_iv.append(iv)
            per_kind.setdefault((_classify(name) or "other") + "+fused", []).append(iv)
            comp_iv.append(iv)
            n_comp += 1
        elif _is_collective(name):
            comm_iv.append(iv)
            per_kind.setdefault(_classify(name) or "other", []).append(iv)
            n_comm += 1
        else:
            comp_iv.append(iv)
            n_comp += 1

    comm_m, comp_m = _merge(comm_iv), _merge(comp_iv)
    if not use_device:
        comp_m = _subtract(comp_m, comm_m)
    everything = _merge(comm_iv + comp_iv)
    wall = (everything[-1][1] - everything[0][0]) if everything else 0.0
    return OverlapReport(
        device=device,
        wall_s=wall,
        compute_s=_total(comp_m),
        comm_s=_total(comm_m),
        overlapped_s=_total(_intersect(comm_m, comp_m)),
        fused_s=_total(_merge(fused_iv)),
        num_comm_events=n_comm,
        num_compute_events=n_comp,
        per_kind_s={k: _total(_merge(v)) for k, v in per_kind.items()},
        note=note,
    )
