"""The fused B200 GPT path (bf16, hand-written kernels) against the portable float32 path."""

from __future__ import annotations

import copy

import pytest
import torch

from minidist.models import GPT, GPTConfig
from minidist.ops import _native as nat

pytestmark = pytest.mark.gpu

CFG = GPTConfig(vocab_size=1000, block_size=256, n_layer=2, n_head=4, n_embd=256)


def _data(B=4, S=256):
    g = torch.Generator().manual_seed(0)
    ids = torch.randint(0, CFG.vocab_size, (B, S), generator=g).cuda()
    tgt = torch.randint(0, CFG.vocab_size, (B, S), generator=g).cuda()
    return ids, tgt


def test_fused_forward_backward_matches_fp32():
    torch.manual_seed(0)
    ref = GPT(CFG, device="cuda")
    fused = copy.deepcopy(ref)
    ids, tgt = _data()
    _, loss_ref = ref(ids, tgt)
    loss_ref.backward()
    with torch.autocast("cuda", dtype=torch.bfloat16):
        logits, loss = fused(ids, tgt)
    assert logits.dtype == torch.bfloat16
    loss.backward()
    nat.check_status()
    assert abs(loss.item() - loss_ref.item()) < 2e-2 * abs(loss_ref.item())
    for (n, p), (_, q) in zip(fused.named_parameters(), ref.named_parameters()):
        assert p.grad is not None, n
        err = ((p.grad - q.grad).abs().max() / q.grad.abs().max().clamp(min=1e-8)).item()
        assert err < 6e-2, f"{n}: rel err {err:.3e}"


def test_fused_training_reduces_loss_and_accumulates():
    from minidist.optim import FusedAdamW

    torch.manual_seed(1)
    model = GPT(CFG, device="cuda")
    opt = FusedAdamW(model.parameters(), lr=1e-3)
    ids, tgt = _data()
    losses = []
    for _ in range(8):
        opt.zero_grad(set_to_none=True)
        with torch.autocast("cuda", dtype=torch.bfloat16):
            _, loss = model(ids, tgt)
        loss.backward()
        opt.step()
        losses.append(loss.item())
    nat.check_status()
    assert losses[-1] < losses[0] - 0.5, losses
    # Two half-batch backwards accumulate to the full-batch gradient.
    opt.zero_grad(set_to_none=True)
    with torch.autocast("cuda", dtype=torch.bfloat16):
        model(ids, tgt)[1].backward()
    full = {n: p.grad.clone() for n, p in model.named_parameters()}
    opt.zero_grad(set_to_none=True)
    for i, t in zip(ids.chunk(2), tgt.chunk(2)):
        with torch.autocast("cuda", dtype=torch.bfloat16):
            (model(i, t)[1] / 2).backward()
    for n, p in model.named_parameters():
        err = ((p.grad - full[n]).abs().max() / full[n].abs().max().clamp(min=1e-8)).item()
        assert err < 3e-2, f"{n}: {err:.3e}"
