"""Fixed-seed determinism runs: the same inputs through the same kernels twice, compared bit for bit.

Which results are bit-identical run to run is part of the kernels' contract:

* GEMM forward / data gradient, LayerNorm forward / backward (dgamma / dbeta reduced in a
  fixed order), column sums, attention forward, and the attention backward's dK / dV (each key
  tile is owned by one CTA) are deterministic;
* the weight gradient with split-K is deterministic only with ``MINIDIST_DETERMINISTIC=1``
  (fixed-order workspace reduction instead of TMA reduce-adds), checked in a subprocess because
  the switch is read at import;
* the attention backward's dQ (reduce-adds from every key tile) and the token-embedding gradient
  (atomics) may differ in the last bits: they are held to fp32 rounding noise instead.
"""

from __future__ import annotations

import os
import subprocess
import sys

import pytest
import torch

from minidist.ops import _native as nat
from minidist.ops import gemm as G
from minidist.ops import kernels as K

pytestmark = pytest.mark.gpu


def _twice(fn):
    a = fn()
    b = fn()
    torch.cuda.synchronize()
    nat.check_status()
    return a, b


def test_deterministic_kernels_are_bit_identical():
    torch.manual_seed(0)
    M, N, Kd = 4096, 2304, 768
    x = torch.randn(M, Kd, device="cuda").bfloat16()
    w = (torch.randn(N, Kd, device="cuda") * 0.02).bfloat16()
    bias = torch.randn(N, device="cuda")
    a, b = _twice(lambda: G.linear_fwd(x, w, bias).clone())
    assert torch.equal(a, b)
    dy = torch.randn(M, N, device="cuda").bfloat16()
    a, b = _twice(lambda: G.linear_dgrad(dy, w).clone())
    assert torch.equal(a, b)
    g, bt = torch.randn(Kd, device="cuda"), torch.randn(Kd, device="cuda")
    a, b = _twice(lambda: K.layernorm_fwd(x, g, bt)[0].clone())
    assert torch.equal(a, b)
    y, mu, rs = K.layernorm_fwd(x, g, bt)

    def ln_bwd():
        dg, db = torch.zeros(Kd, device="cuda"), torch.zeros(Kd, device="cuda")
        dx = K.layernorm_bwd(x, x, mu, rs, g, dgamma=dg, dbeta=db)
        return torch.cat([dx.float().reshape(-1), dg, db])

    a, b = _twice(ln_bwd)
    assert torch.equal(a, b)
    a, b = _twice(lambda: K.colsum(dy, torch.zeros(N, device="cuda")).clone())
    assert torch.equal(a, b)


@pytest.mark.parametrize("D", [64, 128])
def test_attention_run_to_run(D):
    torch.manual_seed(1)
    B, S, H = 2, 1024, 8
    qkv = torch.randn(B * S, 3 * H * D, device="cuda").bfloat16()
    (y1, l1), (y2, l2) = _twice(lambda: tuple(t.clone() for t in K.attention_fwd(qkv, B, S, H, D)))
    assert torch.equal(y1, y2) and torch.equal(l1, l2)
    dy = torch.randn_like(y1)
    g1, g2 = _twice(lambda: K.attention_bwd(qkv, y1, dy, l1, B, S, H, D).clone())
    v1, v2 = (g.view(B * S, H, 3, D) for g in (g1, g2))
    assert torch.equal(v1[:, :, 1:], v2[:, :, 1:])  # dK, dV
    dq = (v1[:, :, 0].float() - v2[:, :, 0].float()).abs().max().item()
    assert dq <= 1e-2 * v1[:, :, 0].float().abs().max().item()  # dQ: accumulation order only


_SPLITK = r"""
import torch
from minidist.ops import gemm as G
torch.manual_seed(2)
dy = torch.randn(8192, 768, device="cuda").bfloat16()
x = torch.randn(8192, 3072, device="cuda").bfloat16()
outs = []
for _ in range(2):
    out = torch.zeros(768, 3072, device="cuda")
    G.linear_wgrad(dy, x, out, k_splits=8)
    outs.append(out)
torch.cuda.synchronize()
assert torch.equal(outs[0], outs[1]), (outs[0] - outs[1]).abs().max().item()
print("ok")
"""


def test_split_k_weight_gradient_deterministic_mode():
    env = dict(os.environ, MINIDIST_DETERMINISTIC="1")
    proc = subprocess.run([sys.executable, "-c", _SPLITK], env=env, capture_output=True, text=True, timeout=300,
                          cwd=os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
    assert proc.returncode == 0 and "ok" in proc.stdout, proc.stdout[-2000:] + proc.stderr[-2000:]
