"""The trainer's B200 path on one GPU: ``--precision bf16 --cuda-graph`` runs the whole step as a
replayed CUDA graph with FusedAdamW(capturable=True) and reports device-timed throughput."""

from __future__ import annotations

import json
import os
import subprocess
import sys

import pytest

pytestmark = pytest.mark.gpu
ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def test_trainer_cuda_graph_step(tmp_path):
    metrics = tmp_path / "m.jsonl"
    cmd = [sys.executable, os.path.join(ROOT, "examples", "train_gpt.py"), "--precision", "bf16", "--cuda-graph",
           "--layers", "2", "--embd", "256", "--heads", "4", "--vocab", "4096", "--seq-len", "256",
           "--batch-size", "8", "--steps", "6", "--metrics-jsonl", str(metrics)]
    proc = subprocess.run(cmd, capture_output=True, text=True, timeout=300, cwd=ROOT)
    assert proc.returncode == 0, proc.stdout[-2000:] + proc.stderr[-3000:]
    recs = [json.loads(line) for line in metrics.read_text().splitlines()]
    summary = [r for r in recs if r.get("event") == "summary"][0]
    assert summary["tokens_per_s"] > 0 and "device" in summary["timing"]
    losses = [r["loss"] for r in recs if "loss" in r]
    assert losses and all(7.0 < v < 9.5 for v in losses), losses  # ~ln(4096) = 8.3 for random tokens
