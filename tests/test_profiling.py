"""Interval arithmetic behind the overlap report, on hand-built traces."""

from __future__ import annotations

import json

import pytest

from minidist.profiling import _intersect, _merge, _subtract, _total, analyze_trace


def test_merge():
    assert _merge([(0, 2), (1, 3), (5, 6)]) == [(0, 3), (5, 6)]
    assert _merge([(0, 1), (1, 2)]) == [(0, 2)]
    assert _merge([]) == []


def test_intersect():
    assert _intersect([(0, 10)], [(2, 4), (6, 12)]) == [(2, 4), (6, 10)]
    assert _intersect([(0, 1)], [(2, 3)]) == []


def test_subtract():
    assert _subtract([(0, 10)], [(2, 4)]) == [(0, 2), (4, 10)]
    assert _subtract([(0, 10)], [(0, 10)]) == []
    assert _subtract([(0, 10)], []) == [(0, 10)]
    assert _total(_subtract([(0, 10)], [(0, 3), (7, 10)])) == 4


def _trace(tmp_path, events):
    p = tmp_path / "t.json"
    p.write_text(json.dumps({"traceEvents": events}))
    return p


def _k(name, ts, dur):
    return {"ph": "X", "cat": "kernel", "name": name, "ts": ts, "dur": dur}


def test_fully_overlapped(tmp_path):
    r = analyze_trace(_trace(tmp_path, [_k("gemm", 0, 1000), _k("nccl:all_reduce", 200, 400)]))
    assert r.device == "cuda" and r.comm_s == pytest.approx(400e-6)
    assert r.overlap_fraction == 1.0 and r.exposed_comm_s == 0.0


def test_fully_exposed(tmp_path):
    r = analyze_trace(_trace(tmp_path, [_k("gemm", 0, 500), _k("nccl:all_gather", 500, 500)]))
    assert r.overlapped_s == 0.0 and r.exposed_comm_s == pytest.approx(500e-6)
    assert r.exposed_fraction_of_step == pytest.approx(0.5)


def test_partial_overlap_and_classification(tmp_path):
    r = analyze_trace(_trace(tmp_path, [_k("gemm", 0, 600), _k("nccl:all_reduce", 400, 400),
                                        _k("ncclDevKernel_ReduceScatter", 800, 100)]))
    assert r.comm_s == pytest.approx(500e-6) and r.overlapped_s == pytest.approx(200e-6)
    assert set(r.per_kind_s) == {"all_reduce", "reduce_scatter"}
    assert r.per_kind_s["reduce_scatter"] == pytest.approx(100e-6)


def test_concurrent_kernels_not_double_counted(tmp_path):
    r = analyze_trace(_trace(tmp_path, [_k("a", 0, 1000), _k("b", 0, 1000)]))
    assert r.compute_s == pytest.approx(1000e-6)


def test_cpu_fallback_is_labelled(tmp_path):
    r = analyze_trace(_trace(tmp_path, [
        {"ph": "X", "cat": "cpu_op", "name": "aten::mm", "ts": 0, "dur": 500},
        {"ph": "X", "cat": "cpu_op", "name": "c10d::allreduce_", "ts": 500, "dur": 300},
    ]))
    assert r.device == "cpu" and "Gloo" in r.note
    assert r.comm_s == pytest.approx(300e-6) and r.overlapped_s == 0.0
    assert "exposed comm" in r.format()


def test_fused_kernels_are_attributed(tmp_path):
    """A fused GEMM+reduce-scatter kernel counts as fused work, not exposed communication."""
    r = analyze_trace(_trace(tmp_path, [_k("void md::md_gemm_rs_kernel<1>(...)", 0, 800),
                                        _k("nccl:all_reduce", 800, 200)]))
    assert r.fused_s == pytest.approx(800e-6)
    assert "reduce_scatter+fused" in r.per_kind_s
    assert r.exposed_comm_s == pytest.approx(200e-6)
