"""Multi-GPU tier on 2, 4 and 8 GPUs (skipped with fewer): peer-memory collectives, the fused GEMM +
all-reduce, DDP, FSDP (gradients and four training steps against DDP), tensor-parallel GPT and its
embedding gather, CUDA-graph replay, GPipe / 1F1B pipelines and tp2 x pp2 x dp composition.

Each test launches ``torchrun`` with one process per GPU (NCCL, 127.0.0.1) on a
worker script in this directory and checks its exit code; the workers assert
the numerics themselves.
"""

from __future__ import annotations

import os
import subprocess
import sys

import pytest
import torch

pytestmark = pytest.mark.gpu

HERE = os.path.dirname(os.path.abspath(__file__))


def _ngpus() -> int:
    return torch.cuda.device_count() if torch.cuda.is_available() else 0


def _torchrun(script: str, n: int, *args: str, timeout: int = 300) -> None:
    env = dict(os.environ, NCCL_NVLS_ENABLE="0", MINIDIST_PEER_TIMEOUT_S="20", PYTHONPATH=os.path.dirname(HERE))
    cmd = ["timeout", "-k", "30", str(timeout), sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
           f"--nproc-per-node={n}", "--master-addr=127.0.0.1", "--master-port=29533",
           os.path.join(HERE, script), *args]
    proc = subprocess.run(cmd, env=env, capture_output=True, text=True)
    assert proc.returncode == 0, proc.stdout[-4000:] + proc.stderr[-4000:]


@pytest.mark.skipif(_ngpus() < 2, reason="needs 2 GPUs")
def test_peer_allreduce_and_ddp_2gpu():
    _torchrun("mgpu_worker.py", 2)


@pytest.mark.skipif(_ngpus() < 4, reason="needs 4 GPUs")
def test_peer_allreduce_and_ddp_4gpu():
    _torchrun("mgpu_worker.py", 4)


@pytest.mark.skipif(_ngpus() < 8, reason="needs 8 GPUs")
def test_peer_allreduce_and_ddp_8gpu():
    _torchrun("mgpu_worker.py", 8, timeout=600)
