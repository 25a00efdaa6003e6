"""Where a training step's device time goes: fused kernels, library collectives, compute.

The reference's profiling layer (profiling.py) answers one question -- how much
communication is *exposed*, i.e. runs with nothing else on the device.  On the
B200 path most communication lives inside fused kernels that do math and
NVLink traffic together, so that question alone undercounts it.  This module
keeps the reference's entry points and report fields and builds them on three
parts of its own:

* **Classes.**  Every device event is ``fused`` (a kernel of this framework
  that moves data between GPUs while it computes -- the ``md_gemm_ar``,
  ``md_ar_bucket``, ``md_rs_shard``, ``md_ag_shards``, ``md_ce_tp`` and
  ``md_embed_tp`` kernels), ``comm`` (a library collective: NCCL kernels,
  ``c10d::`` operators) or ``compute`` (everything else).  :func:`event_class`
  and :func:`collective_kind` hold the name rules.
* **One sweep over the timeline.**  :func:`sweep` walks the sorted start / end
  points of all events once and returns, for every combination of classes,
  how long exactly that combination was active.  Busy time, overlap, exposed
  communication and per-collective time are sums over that table, so
  concurrent kernels are never double-counted and no pairwise interval
  algebra is needed.
* **Peer-wait counters.**  The fused kernels can count, on the device, the
  nanoseconds their CTAs spent waiting for peer GPUs and the nanoseconds they
  ran (:class:`PeerWaitCounters`; ``profile_steps(peer_wait=True)``), which
  splits a fused kernel's time into waiting and working -- something a trace
  of kernel start and end times cannot show.

On a Gloo/CPU trace there are no kernels; the analysis uses CPU operators,
where a collective is a blocking call nested in its caller, so time under a
collective counts as communication only (reference profiling.py:295-361 does
the same by subtraction).
"""

from __future__ import annotations

import gzip
import json
from collections import Counter, defaultdict
from collections.abc import Callable, Iterable, Sequence
from dataclasses import dataclass, field
from pathlib import Path

import torch
from torch.profiler import ProfilerActivity, profile, schedule

__all__ = [
    "COLLECTIVE_PATTERNS",
    "FUSED_KERNELS",
    "OverlapReport",
    "CollectiveRow",
    "KernelRow",
    "PeerWaitCounters",
    "profile_steps",
    "summarize_collectives",
    "format_collective_table",
    "kernel_table",
    "format_kernel_table",
    "analyze_trace",
    "event_class",
    "collective_kind",
    "sweep",
]

# Name fragments of library collectives (NCCL kernels, torch.distributed operators).
COLLECTIVE_PATTERNS: tuple[str, ...] = ("nccl", "c10d::", "record_param_comms", "processgroupnccl",
                                        "processgroupgloo")

# This framework's fused compute + collective kernels: name fragment -> the collective inside.
FUSED_KERNELS: dict[str, str] = {
    "md_gemm_ar": "all_reduce",
    "md_gemm_rs": "reduce_scatter",
    "md_ag_gemm": "all_gather",
    "md_ar_bucket": "all_reduce",
    "md_rs_shard": "reduce_scatter",
    "md_ag_shards": "all_gather",
    "md_ce_tp": "all_reduce",
    "md_embed_tp": "all_gather",
}

# Collective kind from words that appear in NCCL kernel and c10d operator names.
_KIND_WORDS: tuple[tuple[str, tuple[str, ...]], ...] = (
    ("reduce_scatter", ("reducescatter", "reduce_scatter")),
    ("all_gather", ("allgather", "all_gather")),
    ("all_reduce", ("allreduce", "all_reduce")),
    ("broadcast", ("broadcast",)),
    ("send_recv", ("sendrecv", "send", "recv", "p2p")),
    ("barrier", ("barrier",)),
)


def event_class(name: str) -> str:
    """``'fused'``, ``'comm'`` or ``'compute'`` for an event name."""
    low = name.lower()
    if any(frag in low for frag in FUSED_KERNELS):
        return "fused"
    if any(p in low for p in COLLECTIVE_PATTERNS):
        return "comm"
    return "compute"


def collective_kind(name: str) -> str | None:
    """The collective an event performs (``None`` for pure compute)."""
    low = name.lower()
    for frag, kind in FUSED_KERNELS.items():
        if frag in low:
            return kind
    if not any(p in low for p in COLLECTIVE_PATTERNS):
        return None
    for kind, words in _KIND_WORDS:
        if any(w in low for w in words):
            return kind
    return "other"


# ---------------------------------------------------------------------------
# Timeline sweep
# ---------------------------------------------------------------------------

Span = tuple[float, float, str]  # (begin, end, label)


def sweep(spans: Iterable[Span]) -> dict[frozenset, float]:
    """Seconds during which exactly each set of labels was active (idle time is not listed).

    One pass over the 2N sorted boundary points with a count of open spans per
    label; at equal times ends are processed before starts, so touching spans
    do not overlap.
    """
    points: list[tuple[float, int, str]] = []
    for b, e, label in spans:
        if e > b:
            points.append((b, 1, label))
            points.append((e, -1, label))
    points.sort(key=lambda p: (p[0], p[1]))
    open_count: Counter = Counter()
    out: dict[frozenset, float] = defaultdict(float)
    prev = None
    for t, delta, label in points:
        if prev is not None and t > prev:
            active = frozenset(lbl for lbl, n in open_count.items() if n > 0)
            if active:
                out[active] += t - prev
        open_count[label] += delta
        prev = t
    return dict(out)


def _time_where(table: dict[frozenset, float], pred: Callable[[frozenset], bool]) -> float:
    return sum(sec for labels, sec in table.items() if pred(labels))


def busy_time(spans: Iterable[Span]) -> float:
    """Length of the union of the spans."""
    return sum(sweep((b, e, "x") for b, e, _ in spans).values())


# ---------------------------------------------------------------------------
# Running the profiler
# ---------------------------------------------------------------------------


class PeerWaitCounters:
    """Device-side wait / run time of the fused peer-memory kernels.

    While enabled, every CTA of a fused kernel adds to two counters of its
    kernel family: the nanoseconds from its start to its exit (``run``) and
    the nanoseconds it spent spinning on peer GPUs' flags (``wait``).  The
    ratio is the part of the fused kernel's time that went to waiting for
    other ranks (a late peer, or link bandwidth) rather than to its own work.
    Use as a context manager around the steps to measure; :attr:`result`
    holds ``{family: {"wait_ms", "run_ms", "wait_frac", "launches"}}`` with
    times summed over CTAs.
    """

    def __init__(self):
        self.result: dict[str, dict[str, float]] = {}

    def __enter__(self):
        from .ops import _native as nat

        nat.peer_wait_counters(enable=True, reset=True)
        return self

    def __exit__(self, *exc):
        from .ops import _native as nat

        torch.cuda.synchronize()
        self.result = nat.peer_wait_counters(enable=False)
        return False

    def format(self) -> str:
        if not self.result:
            return "  (no fused peer-memory kernel ran)"
        lines = [f"  {'fused kernel':<16}{'launches':>9}{'CTA-ms run':>12}{'CTA-ms wait':>13}{'waiting':>9}"]
        for fam, r in sorted(self.result.items(), key=lambda kv: -kv[1]["run_ms"]):
            lines.append(f"  {fam:<16}{int(r['launches']):>9}{r['run_ms']:>12.2f}{r['wait_ms']:>13.2f}"
                         f"{r['wait_frac'] * 100:>8.1f}%")
        return "\n".join(lines)


def profile_steps(
    step_fn: Callable[[int], None],
    num_steps: int = 6,
    warmup: int = 2,
    wait: int = 1,
    trace_path: str | Path | None = None,
    record_shapes: bool = True,
    with_stack: bool = False,
    activities: Sequence[ProfilerActivity] | None = None,
    peer_wait: bool = False,
):
    """Run ``step_fn(step)`` ``num_steps`` times under ``torch.profiler`` and return the profiler.

    The first ``wait`` steps are not recorded and the next ``warmup`` are
    recorded and dropped, so one-off costs (communicator set-up, allocator
    growth, lazy kernel attributes) stay out of the measured steps.  With
    ``trace_path`` a Chrome trace is written there.  With ``peer_wait`` (CUDA
    only) the measured steps also run under :class:`PeerWaitCounters`; the
    result is attached to the returned profiler as ``md_peer_wait``.
    """
    if activities is None:
        activities = [ProfilerActivity.CPU] + ([ProfilerActivity.CUDA] if torch.cuda.is_available() else [])
    active = max(1, num_steps - wait - warmup)
    counters = PeerWaitCounters() if (peer_wait and torch.cuda.is_available()) else None
    with profile(activities=list(activities), schedule=schedule(wait=wait, warmup=warmup, active=active, repeat=1),
                 record_shapes=record_shapes, with_stack=with_stack, profile_memory=True) as prof:
        for step in range(num_steps):
            if counters is not None and step == wait + warmup:
                counters.__enter__()
            step_fn(step)
            prof.step()
    if counters is not None:
        counters.__exit__(None, None, None)
    prof.md_peer_wait = counters
    if trace_path is not None:
        trace_path = Path(trace_path)
        trace_path.parent.mkdir(parents=True, exist_ok=True)
        prof.export_chrome_trace(str(trace_path))
    return prof


# ---------------------------------------------------------------------------
# Event-table summaries
# ---------------------------------------------------------------------------


@dataclass
class CollectiveRow:
    """Totals of one collective kind (``<kind>+fused`` for the fused kernels)."""

    kind: str
    count: int
    self_time_us: float
    device_time_us: float
    fused: bool = False

    @property
    def avg_us(self) -> float:
        return (self.device_time_us or self.self_time_us) / max(1, self.count)


def _device_us(evt) -> float:
    for attr in ("self_device_time_total", "self_cuda_time_total"):
        v = getattr(evt, attr, None)
        if v:
            return float(v)
    return 0.0


def summarize_collectives(prof) -> list[CollectiveRow]:
    """Per-collective-kind totals from a profiler's event table, largest first."""
    rows: dict[str, CollectiveRow] = {}
    for evt in prof.key_averages():
        cls = event_class(evt.key)
        if cls == "compute":
            continue
        fused = cls == "fused"
        kind = (collective_kind(evt.key) or "other") + ("+fused" if fused else "")
        row = rows.get(kind) or rows.setdefault(kind, CollectiveRow(kind, 0, 0.0, 0.0, fused))
        row.count += evt.count
        row.self_time_us += float(getattr(evt, "self_cpu_time_total", 0.0) or 0.0)
        row.device_time_us += _device_us(evt)
    return sorted(rows.values(), key=lambda r: (r.device_time_us, r.self_time_us), reverse=True)


def format_collective_table(rows: Iterable[CollectiveRow]) -> str:
    rows = list(rows)
    if not rows:
        return "  (no collective ran in the measured steps)"
    head = f"  {'kind':<24}{'calls':>7}{'device ms':>11}{'host ms':>10}{'us/call':>10}"
    body = [f"  {r.kind:<24}{r.count:>7}{r.device_time_us / 1e3:>11.2f}{r.self_time_us / 1e3:>10.2f}"
            f"{r.avg_us:>10.1f}" for r in rows]
    return "\n".join([head, *body])


@dataclass
class KernelRow:
    """One device kernel's totals and its class (fused / comm / compute)."""

    name: str
    cls: str
    count: int
    device_time_us: float
    share: float = 0.0


def kernel_table(prof_or_trace, top: int = 20) -> list[KernelRow]:
    """The ``top`` kernels by device time, from a profiler object or a Chrome-trace path, each with
    its class and its share of all kernel time -- the per-fused-kernel attribution of a step."""
    acc: dict[str, list] = {}
    if isinstance(prof_or_trace, (str, Path)):
        for e in _kernel_events(_load_trace(prof_or_trace)):
            a = acc.setdefault(e["name"], [0, 0.0])
            a[0] += 1
            a[1] += float(e.get("dur", 0.0))
    else:
        for evt in prof_or_trace.key_averages():
            us = _device_us(evt)
            if us > 0:
                a = acc.setdefault(evt.key, [0, 0.0])
                a[0] += evt.count
                a[1] += us
    total = sum(a[1] for a in acc.values()) or 1.0
    rows = [KernelRow(n, event_class(n), a[0], a[1], a[1] / total) for n, a in acc.items()]
    rows.sort(key=lambda r: r.device_time_us, reverse=True)
    return rows[:top]


def format_kernel_table(rows: Iterable[KernelRow], width: int = 60) -> str:
    lines = [f"  {'kernel':<{width}}{'class':>9}{'calls':>7}{'ms':>9}{'share':>8}"]
    for r in rows:
        name = r.name if len(r.name) <= width else r.name[: width - 3] + "..."
        lines.append(f"  {name:<{width}}{r.cls:>9}{r.count:>7}{r.device_time_us / 1e3:>9.2f}{r.share * 100:>7.1f}%")
    return "\n".join(lines)


# ---------------------------------------------------------------------------
# Trace analysis
# ---------------------------------------------------------------------------


@dataclass
class OverlapReport:
    """Device (or CPU) time of one trace by class, in seconds.

    ``comm_s`` is library-collective time, ``overlapped_s`` the part of it that
    ran beside compute or a fused kernel, ``fused_s`` the time any fused
    compute + collective kernel was running (its communication is hidden
    inside it by construction), ``wall_s`` first start to last end.
    """

    device: str
    wall_s: float = 0.0
    compute_s: float = 0.0
    comm_s: float = 0.0
    overlapped_s: float = 0.0
    fused_s: float = 0.0
    idle_s: float = 0.0
    num_comm_events: int = 0
    num_compute_events: int = 0
    num_fused_events: int = 0
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

    def as_dict(self) -> dict:
        d = {k: getattr(self, k) for k in ("device", "wall_s", "compute_s", "comm_s", "overlapped_s", "fused_s",
                                             "idle_s", "num_comm_events", "num_compute_events", "num_fused_events")}
        d.update(exposed_comm_s=self.exposed_comm_s, overlap_fraction=self.overlap_fraction,
                 exposed_fraction_of_step=self.exposed_fraction_of_step, per_kind_s=dict(self.per_kind_s))
        return d

    def format(self) -> str:
        ms = lambda s: f"{s * 1e3:9.2f} ms"  # noqa: E731
        pct = lambda a, b: f"{(a / b * 100 if b else 0.0):5.1f}%"  # noqa: E731
        rows = [
            ("timeline", ms(self.wall_s), f"{self.device} events, first start to last end"),
            ("compute", ms(self.compute_s), f"{self.num_compute_events} events"),
            ("fused comm+compute", ms(self.fused_s), f"{self.num_fused_events} events, "
                                                      f"{pct(self.fused_s, self.wall_s)} of timeline"),
            ("library comm", ms(self.comm_s), f"{self.num_comm_events} events"),
            ("  hidden by compute", ms(self.overlapped_s), pct(self.overlapped_s, self.comm_s) + " of library comm"),
            ("  exposed", ms(self.exposed_comm_s), pct(self.exposed_comm_s, self.wall_s) + " of timeline"),
            ("idle", ms(self.idle_s), pct(self.idle_s, self.wall_s) + " of timeline"),
        ]
        lines = [f"  {a:<22}{b}   {c}" for a, b, c in rows]
        for kind, sec in sorted(self.per_kind_s.items(), key=lambda kv: -kv[1]):
            lines.append(f"    {kind:<20}{ms(sec)}")
        if self.note:
            lines.append(f"  note: {self.note}")
        return "\n".join(lines)


def _load_trace(path: str | Path) -> dict:
    path = Path(path)
    with (gzip.open(path, "rt") if path.suffix == ".gz" else open(path)) as fh:
        return json.load(fh)


def _kernel_events(trace: dict) -> list[dict]:
    return [e for e in trace.get("traceEvents", []) if e.get("ph") == "X" and e.get("cat") == "kernel"]


def analyze_trace(path: str | Path, prefer_device: bool = True) -> OverlapReport:
    """Time by class (compute / fused / library comm), overlap and exposed communication of a Chrome trace.

    Uses GPU kernels when the trace has them, else CPU operators (Gloo / CPU runs).
    """
    trace = _load_trace(path)
    kernels = _kernel_events(trace) if prefer_device else []
    on_device = bool(kernels)
    if on_device:
        events, device, note = kernels, "cuda", ""
    else:
        events = [e for e in trace.get("traceEvents", [])
                  if e.get("ph") == "X" and e.get("cat") in ("cpu_op", "user_annotation")]
        device = "cpu"
        note = ("CPU trace (Gloo): a collective blocks its caller, so nothing overlaps it here; "
                "measure overlap on a CUDA + NCCL trace")
    spans: list[Span] = []
    kind_spans: list[Span] = []
    counts: Counter = Counter()
    for e in events:
        b = float(e["ts"]) * 1e-6
        end = b + float(e.get("dur", 0.0)) * 1e-6
        name = e.get("name", "")
        cls = event_class(name)
        counts[cls] += 1
        spans.append((b, end, cls))
        if cls != "compute":
            kind_spans.append((b, end, (collective_kind(name) or "other") + ("+fused" if cls == "fused" else "")))
    table = sweep(spans)
    if on_device:
        compute = _time_where(table, lambda s: "compute" in s or "fused" in s)
        overlapped = _time_where(table, lambda s: "comm" in s and ("compute" in s or "fused" in s))
    else:
        # CPU operators nest: the caller of a blocking collective is "busy" while it waits.
        compute = _time_where(table, lambda s: "comm" not in s)
        overlapped = 0.0
    per_kind: dict[str, float] = defaultdict(float)
    for labels, sec in sweep(kind_spans).items():
        for lbl in labels:
            per_kind[lbl] += sec
    busy = sum(table.values())
    wall = (max(e for _, e, _ in spans) - min(b for b, _, _ in spans)) if spans else 0.0
    return OverlapReport(
        device=device,
        wall_s=wall,
        compute_s=compute,
        comm_s=_time_where(table, lambda s: "comm" in s),
        overlapped_s=overlapped,
        fused_s=_time_where(table, lambda s: "fused" in s),
        idle_s=max(0.0, wall - busy),
        num_comm_events=counts["comm"],
        num_compute_events=counts["compute"],
        num_fused_events=counts["fused"],
        per_kind_s=dict(per_kind),
        note=note,
    )
