"""Runs the *reference* package (``baseline/_ref``) for tests/test_reference_parity.py.

Executed as a separate Python process so that the reference's ``minidist``
never shares an interpreter with this repository's.  Modes:

* ``init OUT``            -- GPT(CFG).state_dict() with the test seed -> OUT
* ``loss CKPT OUT``       -- GPT(CFG) loaded from CKPT (a consolidated state dict) -> loss and logits on the
                             fixed batch -> OUT
* ``fsdp OUT`` (torchrun) -- the reference FSDP's named flat shards of every rank -> OUT_rank{r}
"""

from __future__ import annotations

import os
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(os.path.dirname(HERE), "baseline", "_ref"))

import torch  # noqa: E402

import minidist  # noqa: E402
from minidist.models import GPT, Block, GPTConfig  # noqa: E402

assert os.path.realpath(minidist.__file__).startswith(os.path.realpath(os.path.join(os.path.dirname(HERE), "baseline")))

CFG = dict(vocab_size=96, block_size=16, n_layer=3, n_head=4, n_embd=32, seed=77)


def batch():
    g = torch.Generator().manual_seed(5)
    return (torch.randint(0, CFG["vocab_size"], (4, 16), generator=g),
            torch.randint(0, CFG["vocab_size"], (4, 16), generator=g))


def main() -> None:
    mode = sys.argv[1]
    if mode == "init":
        torch.save(GPT(GPTConfig(**CFG)).state_dict(), sys.argv[2])
    elif mode == "loss":
        m = GPT(GPTConfig(**CFG))
        m.load_state_dict(torch.load(sys.argv[2]))
        ids, tgt = batch()
        logits, loss = m(ids, tgt)
        torch.save({"loss": loss.detach(), "logits": logits.detach()}, sys.argv[3])
    elif mode == "fsdp":
        rank, world, _ = minidist.init_distributed(backend="gloo")
        m = minidist.FullyShardedDataParallel(GPT(GPTConfig(**CFG)), unit_types=(Block,))
        torch.save({n: p.detach().clone() for n, p in m.named_parameters()}, f"{sys.argv[2]}_rank{rank}")
        minidist.shutdown_distributed()
    else:
        raise SystemExit(f"unknown mode {mode}")


if __name__ == "__main__":
    main()
