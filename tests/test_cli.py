"""End-to-end CLI checks on Gloo: the trainer and the benchmark scripts run under torchrun."""

from __future__ import annotations

import os
import re
import subprocess
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _torchrun(script: str, n: int, port: int, *args: str) -> str:
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", f"--nproc-per-node={n}",
           "--master-addr=127.0.0.1", f"--master-port={port}", os.path.join(ROOT, script), *args]
    env = dict(os.environ, OMP_NUM_THREADS="1", CUDA_VISIBLE_DEVICES="")
    proc = subprocess.run(cmd, capture_output=True, text=True, timeout=600, env=env, cwd=ROOT)
    assert proc.returncode == 0, proc.stdout[-3000:] + proc.stderr[-3000:]
    return proc.stdout


def test_trainer_3d_parallel_smoke():
    out = _torchrun("examples/train_gpt.py", 4, 29571, "--tp", "2", "--pp", "2", "--strategy", "none",
                    "--microbatches", "4", "--layers", "4", "--embd", "128", "--heads", "4", "--vocab", "1024",
                    "--seq-len", "64", "--batch-size", "8", "--steps", "2", "--backend", "gloo")
    losses = [float(x) for x in re.findall(r"loss\s+([0-9.]+)", out)]
    assert losses and all(6.0 < v < 8.0 for v in losses), out  # ~ln(1024) = 6.93 for random tokens
    assert "pipeline bubble" in out


def test_trainer_ddp_and_fsdp_smoke():
    for strategy in ("ddp", "fsdp"):
        out = _torchrun("examples/train_gpt.py", 2, 29572, "--strategy", strategy, "--layers", "2", "--embd", "64",
                        "--heads", "4", "--vocab", "256", "--seq-len", "32", "--batch-size", "4", "--steps", "2",
                        "--backend", "gloo")
        assert "tok/s" in out


def test_benchmark_scripts_smoke():
    out = _torchrun("benchmarks/bench_parallelism.py", 2, 29573, "--layers", "2", "--embd", "64", "--heads", "4",
                    "--vocab", "256", "--seq-len", "32", "--batch-size", "4", "--iters", "1", "--warmup", "1",
                    "--backend", "gloo")
    assert "speed-ups" in out
    out = _torchrun("benchmarks/bench_pipeline.py", 2, 29574, "--microbatches", "1,2", "--layers", "4", "--embd", "64",
                    "--heads", "4", "--vocab", "256", "--seq-len", "32", "--batch-size", "4", "--iters", "1",
                    "--backend", "gloo", "--gantt")
    assert "stage 0 |" in out and "theory" in out
    out = _torchrun("benchmarks/bench_collectives.py", 2, 29575, "--max-mb", "1", "--iters", "2", "--warmup", "1",
                    "--backend", "gloo")
    assert "all_reduce" in out


def test_trainer_metrics_jsonl_and_kernels_flag(tmp_path):
    import json

    path = tmp_path / "metrics.jsonl"
    _torchrun("examples/train_gpt.py", 2, 29576, "--strategy", "ddp", "--layers", "2", "--embd", "64", "--heads", "4",
              "--vocab", "256", "--seq-len", "32", "--batch-size", "4", "--steps", "3", "--backend", "gloo",
              "--kernels", "nccl", "--metrics-jsonl", str(path))
    recs = [json.loads(line) for line in path.read_text().splitlines()]
    steps = [r for r in recs if "step" in r]
    summary = [r for r in recs if r.get("event") == "summary"]
    assert steps and all(r["loss"] > 0 and r["tokens_per_s"] > 0 for r in steps)
    assert len(summary) == 1 and summary[0]["steps"] == 3 and summary[0]["kernels"] == "nccl"
