"""Interchangeability with the reference package installed under baseline/_ref (CPU).

* equal seeds give bit-identical initial weights in both packages (the reference's
  ``_seed_for`` / ``full_linear_weight`` draws, models/gpt.py:76-77);
* a checkpoint written by this package's ``checkpoint.save`` + ``consolidate`` loads into the
  reference's ``GPT.load_state_dict`` and computes the same loss and logits, and the reference's
  state dict loads into ours;
* FSDP exposes the same ``_flat_shard_{i}`` parameters on every rank (names, padding, contents) as
  the reference's FSDP (fsdp.py:133-151, 411-420), so sharded optimizer state lines up.

The reference runs in its own process (tests/ref_worker.py); nothing here imports it.
"""

from __future__ import annotations

import os
import subprocess
import sys

import pytest
import torch

from minidist.models import GPT, GPTConfig
from minidist.utils import checkpoint

from .harness import run_distributed

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
WORKER = os.path.join(ROOT, "tests", "ref_worker.py")
pytestmark = pytest.mark.skipif(not os.path.isdir(os.path.join(ROOT, "baseline", "_ref", "minidist")),
                                reason="baseline/_ref not installed")
CFG = dict(vocab_size=96, block_size=16, n_layer=3, n_head=4, n_embd=32, seed=77)


def _ref(*args, n: int = 0) -> None:
    env = dict(os.environ, CUDA_VISIBLE_DEVICES="", OMP_NUM_THREADS="1", PYTHONPATH="")
    if n:
        cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", f"--nproc-per-node={n}",
               "--master-addr=127.0.0.1", "--master-port=29655", WORKER, *args]
    else:
        cmd = [sys.executable, WORKER, *args]
    proc = subprocess.run(cmd, capture_output=True, text=True, timeout=300, env=env, cwd="/tmp")
    assert proc.returncode == 0, proc.stdout[-2000:] + proc.stderr[-3000:]


def _batch():
    g = torch.Generator().manual_seed(5)
    return (torch.randint(0, CFG["vocab_size"], (4, 16), generator=g),
            torch.randint(0, CFG["vocab_size"], (4, 16), generator=g))


def test_equal_seeds_give_identical_weights(tmp_path):
    _ref("init", str(tmp_path / "ref.pt"))
    theirs = torch.load(tmp_path / "ref.pt")
    ours = GPT(GPTConfig(**CFG)).state_dict()
    assert list(theirs) == list(ours)
    for k in ours:
        assert torch.equal(ours[k], theirs[k]), k


def test_our_checkpoint_loads_into_the_reference(tmp_path):
    model = GPT(GPTConfig(**CFG))
    with torch.no_grad():
        for i, p in enumerate(model.parameters()):
            p.add_(0.003 * (i + 1))
    checkpoint.save(str(tmp_path / "ck"), model, step=1)
    torch.save(checkpoint.consolidate(str(tmp_path / "ck")), tmp_path / "merged.pt")
    _ref("loss", str(tmp_path / "merged.pt"), str(tmp_path / "out.pt"))
    got = torch.load(tmp_path / "out.pt")
    logits, loss = model(*_batch())
    assert torch.allclose(got["logits"], logits.detach(), atol=1e-6, rtol=1e-5)
    assert abs(got["loss"].item() - loss.item()) < 1e-6


def test_reference_state_dict_loads_into_ours(tmp_path):
    _ref("init", str(tmp_path / "ref.pt"))
    ours = GPT(GPTConfig(**{**CFG, "seed": 1}))
    ours.load_state_dict(torch.load(tmp_path / "ref.pt"))
    _ref("loss", str(tmp_path / "ref.pt"), str(tmp_path / "out.pt"))
    got = torch.load(tmp_path / "out.pt")
    logits, loss = ours(*_batch())
    assert torch.allclose(got["logits"], logits.detach(), atol=1e-6, rtol=1e-5)


def _our_fsdp_shards(rank, world, out):
    from minidist.fsdp import FullyShardedDataParallel
    from minidist.models import Block

    m = FullyShardedDataParallel(GPT(GPTConfig(**CFG)), unit_types=(Block,))
    torch.save({n: p.detach().clone() for n, p in m.named_parameters()}, f"{out}_rank{rank}")


def test_fsdp_flat_shards_match_the_reference(tmp_path):
    _ref("fsdp", str(tmp_path / "ref"), n=2)
    run_distributed(_our_fsdp_shards, 2, str(tmp_path / "ours"))
    for r in range(2):
        theirs = torch.load(f"{tmp_path / 'ref'}_rank{r}")
        ours = torch.load(f"{tmp_path / 'ours'}_rank{r}")
        assert list(theirs) == list(ours)
        for k in ours:
            assert theirs[k].shape == ours[k].shape and torch.equal(theirs[k], ours[k]), (r, k)
