"""bench.py wiring on Gloo/CPU: both arms build every configuration through their own public API.

The reference arm imports the unmodified reference package from ``baseline/_ref``
(skipped where it is not installed) and must accept exactly the reference's
constructor signatures -- a repo-only keyword passed to its DDP once crashed it
at N >= 2.  On the same seeds both arms must report the same loss (fp32 on CPU).
"""

from __future__ import annotations

import json
import os
import subprocess
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HAVE_REF = os.path.isdir(os.path.join(ROOT, "baseline", "_ref", "minidist"))


def _bench(n: int, port: int, *args: str) -> dict:
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", f"--nproc-per-node={n}",
           "--master-addr=127.0.0.1", f"--master-port={port}", os.path.join(ROOT, "bench.py"),
           "--gpus", str(n), "--device", "cpu", "--tiny", "--steps", "2", "--warmup", "1", *args]
    env = dict(os.environ, OMP_NUM_THREADS="1", CUDA_VISIBLE_DEVICES="")
    proc = subprocess.run(cmd, capture_output=True, text=True, timeout=600, env=env, cwd=ROOT)
    assert proc.returncode == 0, proc.stdout[-3000:] + proc.stderr[-3000:]
    lines = [ln for ln in proc.stdout.splitlines() if ln.startswith("{")]
    assert len(lines) == 1, proc.stdout
    return json.loads(lines[0])


@pytest.mark.skipif(not HAVE_REF, reason="baseline/_ref not installed")
@pytest.mark.parametrize("config,n,port", [("gpt2s-ddp", 2, 29641), ("gpt1.5b-fsdp", 2, 29643),
                                           ("gpt2.7b-3d", 4, 29645)])
def test_both_arms_same_loss(config, n, port):
    ref = _bench(n, port, "--impl", "reference", "--config", config)
    ours = _bench(n, port + 1, "--impl", "ours", "--config", config)
    assert ref["impl"] == "reference" and "impl" not in ours
    for out in (ref, ours):
        # The driver's contract: one JSON line with these keys on both arms.
        for key in ("metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step", "higher_is_better",
                    "scaling", "vs_baseline", "dtype", "data", "config", "e2e", "gpu_launches"):
            assert key in out, (key, out)
        for key in ("model", "global_batch", "seq_len", "parallelism"):
            assert key in out["config"], (key, out["config"])
        assert out["metric"] == ref["metric"] and out["higher_is_better"] is True
        assert out["n_gpus"] == n and out["steps"] == 2 and out["warmup"] == 1
        assert out["value"] > 0 and out["e2e"]["value"] > 0
        assert out["config"]["name"] == config
    assert abs(ref["final_loss"] - ours["final_loss"]) < 1e-4 * abs(ref["final_loss"]), (ref, ours)


def test_layout_resolution():
    sys.path.insert(0, ROOT)
    import bench

    c = bench.resolve_config("gpt2.7b-3d", 8)
    assert (c["tp"], c["pp"], c["dp"], c["microbatches"], c["batch"] * c["dp"]) == (2, 2, 2, 8, 64)
    c = bench.resolve_config("gpt6.7b-tp8", 8)
    assert (c["tp"], c["pp"], c["dp"]) == (8, 1, 1)
    c = bench.resolve_config("gpt2s-ddp", 8)
    assert (c["tp"], c["dp"], c["batch"]) == (1, 8, 16)
    with pytest.raises(SystemExit):
        bench.resolve_config("gpt2.7b-3d", 2)


@pytest.mark.skipif(not HAVE_REF, reason="baseline/_ref not installed")
def test_reference_1f1b_on_gpus_reports_unavailable(monkeypatch, capsys):
    """The reference's 1F1B deadlocks on NCCL at this configuration's message sizes, so on
    GPUs its arm prints the one-line ``unavailable`` record (and builds nothing) instead."""
    sys.path.insert(0, ROOT)
    import bench

    monkeypatch.setenv("WORLD_SIZE", "4")
    monkeypatch.setenv("RANK", "0")
    assert bench.main(["--impl", "reference", "--config", "gpt2.7b-3d", "--gpus", "4"]) == 0
    out = json.loads(capsys.readouterr().out.strip().splitlines()[-1])
    assert out["impl"] == "reference" and "deadlocks" in out["unavailable"]
