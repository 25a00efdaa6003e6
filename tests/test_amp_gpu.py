"""The loss scaler's overflow test and unscale folded into the FusedAdamW kernel (CUDA).

An overflow anywhere leaves every weight and moment untouched and halves the
scale; a clean step equals torch.optim.AdamW on the unscaled gradients.
"""

from __future__ import annotations

import pytest
import torch

from minidist.amp import DistributedGradScaler
from minidist.optim import FusedAdamW

pytestmark = pytest.mark.gpu


def _params():
    g = torch.Generator(device="cuda").manual_seed(0)
    return [torch.randn(n, device="cuda", generator=g).requires_grad_(True) for n in (1000, 8192 * 3 + 5, 77)]


def test_overflow_skips_on_device_and_backs_off():
    ps = _params()
    before = [p.detach().clone() for p in ps]
    opt = FusedAdamW(ps, lr=1e-2)
    sc = DistributedGradScaler(init_scale=1024.0)
    for p in ps:
        p.grad = torch.randn_like(p) * 1024
    ps[1].grad[12345] = float("inf")
    assert sc.step(opt) is True  # issued; the kernel decides
    sc.update()
    assert sc.scale == 512.0 and sc.num_skipped == 1
    for p, b in zip(ps, before):
        assert torch.equal(p.detach(), b)
    assert all(float(opt.state[p]["exp_avg"].abs().sum()) == 0.0 for p in ps)


def test_clean_step_matches_torch_adamw_on_unscaled_grads():
    ps, ref = _params(), _params()
    opt = FusedAdamW(ps, lr=1e-2)
    ropt = torch.optim.AdamW(ref, lr=1e-2)
    sc = DistributedGradScaler(init_scale=256.0)
    for it in range(3):
        g = torch.Generator(device="cuda").manual_seed(10 + it)
        for p, r in zip(ps, ref):
            gr = torch.randn(p.shape, device="cuda", generator=g)
            p.grad, r.grad = gr * 256.0, gr.clone()
        sc.step(opt)
        sc.update()
        ropt.step()
    assert sc.num_skipped == 0
    for p, r in zip(ps, ref):
        assert (p.detach() - r.detach()).abs().max().item() < 1e-5
