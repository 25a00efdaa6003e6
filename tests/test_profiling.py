"""Timeline attribution (minidist.profiling) on hand-built Chrome traces.

Cases: classification of event names, the boundary sweep, overlap of library
collectives with compute, fused kernels counted as fused work, concurrency,
idle gaps, the CPU (Gloo) fallback, the per-kernel table and the peer-wait
table's formatting.
"""

from __future__ import annotations

import json

import pytest

from minidist.profiling import (
    PeerWaitCounters,
    analyze_trace,
    busy_time,
    collective_kind,
    event_class,
    format_kernel_table,
    kernel_table,
    sweep,
)


def _trace(tmp_path, events, name="t.json"):
    p = tmp_path / name
    p.write_text(json.dumps({"traceEvents": events}))
    return p


def _k(name, ts, dur):
    return {"ph": "X", "cat": "kernel", "name": name, "ts": ts, "dur": dur}


def test_event_classes_and_kinds():
    assert event_class("ncclDevKernel_AllGather_RING_LL(ncclDevKernelArgsStorage<4096ul>)") == "comm"
    assert collective_kind("ncclDevKernel_AllGather_RING_LL") == "all_gather"
    assert collective_kind("c10d::reduce_scatter_tensor_coalesced_") == "reduce_scatter"
    assert event_class("void md::gemm::md_gemm_ar_kernel<2, 8, false, false, 1>(...)") == "fused"
    assert collective_kind("void md::symm::md_embed_tp_kernel(MdEmbTpParams)") == "all_gather"
    assert collective_kind("void md::symm::md_ar_bucket_kernel(MdArParams)") == "all_reduce"
    assert event_class("void md::attn_tc::fwd_kernel<64>(...)") == "compute"
    assert collective_kind("sm100_xmma_gemm_bf16bf16") is None


def test_sweep_splits_time_by_active_set():
    t = sweep([(0, 4, "a"), (2, 6, "b"), (6, 7, "a")])
    assert t == {frozenset("a"): 3, frozenset("ab"): 2, frozenset("b"): 2}
    assert busy_time([(0, 4, "a"), (2, 6, "b"), (8, 9, "c")]) == 7


def test_sweep_touching_spans_do_not_overlap():
    t = sweep([(0, 1, "a"), (1, 2, "b")])
    assert frozenset("ab") not in t and sum(t.values()) == 2


def test_comm_under_compute_is_hidden(tmp_path):
    r = analyze_trace(_trace(tmp_path, [_k("sm100_gemm", 0, 900), _k("ncclDevKernel_AllReduce", 300, 300)]))
    assert r.device == "cuda" and r.comm_s == pytest.approx(300e-6)
    assert r.overlap_fraction == 1.0 and r.exposed_comm_s == 0.0 and r.idle_s == 0.0


def test_comm_after_compute_is_exposed(tmp_path):
    r = analyze_trace(_trace(tmp_path, [_k("ln_fwd", 0, 300), _k("ncclDevKernel_ReduceScatter", 300, 100),
                                        _k("ncclDevKernel_AllGather", 500, 100)]))
    assert r.exposed_comm_s == pytest.approx(200e-6) and r.overlapped_s == 0.0
    assert r.idle_s == pytest.approx(100e-6)
    assert r.exposed_fraction_of_step == pytest.approx(200 / 600)
    assert r.per_kind_s == pytest.approx({"reduce_scatter": 100e-6, "all_gather": 100e-6})


def test_fused_kernel_hides_library_comm_and_is_reported(tmp_path):
    r = analyze_trace(_trace(tmp_path, [
        _k("void md::gemm::md_gemm_ar_kernel<1, 8, false, false, 1>(...)", 0, 700),
        _k("ncclDevKernel_SendRecv", 600, 200),
        _k("attn_fwd", 800, 100),
    ]))
    assert r.fused_s == pytest.approx(700e-6) and r.num_fused_events == 1
    assert r.overlapped_s == pytest.approx(100e-6) and r.exposed_comm_s == pytest.approx(100e-6)
    assert r.per_kind_s["all_reduce+fused"] == pytest.approx(700e-6)
    assert r.per_kind_s["send_recv"] == pytest.approx(200e-6)
    assert "fused comm+compute" in r.format()


def test_three_concurrent_streams_counted_once(tmp_path):
    r = analyze_trace(_trace(tmp_path, [_k("a", 0, 1000), _k("b", 100, 800), _k("c", 200, 100)]))
    assert r.compute_s == pytest.approx(1000e-6) and r.wall_s == pytest.approx(1000e-6)


def test_cpu_trace_counts_blocking_collectives_as_comm(tmp_path):
    r = analyze_trace(_trace(tmp_path, [
        {"ph": "X", "cat": "cpu_op", "name": "ProfilerStep#3", "ts": 0, "dur": 1000},
        {"ph": "X", "cat": "cpu_op", "name": "aten::addmm", "ts": 50, "dur": 400},
        {"ph": "X", "cat": "cpu_op", "name": "c10d::allreduce_", "ts": 500, "dur": 300},
    ]))
    assert r.device == "cpu" and "Gloo" in r.note
    assert r.comm_s == pytest.approx(300e-6) and r.overlapped_s == 0.0
    assert r.compute_s == pytest.approx(700e-6) and r.exposed_comm_s == pytest.approx(300e-6)


def test_kernel_table_shares(tmp_path):
    p = _trace(tmp_path, [_k("gemm", 0, 600), _k("gemm", 700, 200), _k("void md::symm::md_rs_shard_kernel(x)", 0, 200)])
    rows = kernel_table(p)
    assert [r.name for r in rows] == ["gemm", "void md::symm::md_rs_shard_kernel(x)"]
    assert rows[0].count == 2 and rows[0].share == pytest.approx(0.8) and rows[1].cls == "fused"
    assert "md_rs_shard" in format_kernel_table(rows)


def test_peer_wait_table_format():
    c = PeerWaitCounters()
    assert "no fused" in c.format()
    c.result = {"md_ar_bucket": {"run_ms": 10.0, "wait_ms": 2.5, "wait_frac": 0.25, "launches": 12}}
    out = c.format()
    assert "md_ar_bucket" in out and "25.0%" in out
