"""The bounds-checking build (``python -m minidist._build --bounds-check``, loaded with
``MINIDIST_BOUNDS_CHECK=1``): a clean training step reports nothing and computes what the normal
build computes; a token id outside the vocabulary is reported (site, value) through the status
word instead of being silently treated as a zero row.  Runs in subprocesses, since the library
choice is made at import."""

from __future__ import annotations

import os
import subprocess
import sys

import pytest

pytestmark = pytest.mark.gpu
ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))

_STEP = r"""
import torch
from minidist.models import GPT, GPTConfig
from minidist.ops import _native as nat
cfg = GPTConfig(vocab_size=4096, block_size=256, n_layer=2, n_head=12, n_embd=768)
torch.manual_seed(0)
model = GPT(cfg, device="cuda")
g = torch.Generator().manual_seed(1)
ids = torch.randint(0, 4096, (2, 256), generator=g).cuda()
with torch.autocast("cuda", dtype=torch.bfloat16):
    _, loss = model(ids, ids)
loss.backward()
nat.check_status()
print("LOSS", repr(float(loss)), "CHECKED", nat.bounds_checked())
"""

_BAD_ID = r"""
import torch
from minidist.ops import _native as nat, kernels as K
wte = torch.randn(1000, 64, device="cuda").bfloat16()
ids = torch.tensor([[3, -7, 5]], device="cuda")
K.embedding_fwd(ids, wte, None, 3)
try:
    nat.check_status()
    print("NOT REPORTED")
except nat.NativeError as e:
    print("REPORTED", e)
"""


def _run(code: str, checked: bool) -> str:
    env = dict(os.environ, MINIDIST_BOUNDS_CHECK="1" if checked else "0")
    proc = subprocess.run([sys.executable, "-c", code], env=env, cwd=ROOT, capture_output=True, text=True, timeout=300)
    assert proc.returncode == 0, proc.stdout[-2000:] + proc.stderr[-3000:]
    return proc.stdout


@pytest.mark.skipif(not os.path.exists(os.path.join(ROOT, "minidist", "_lib", "libminidist_cuda_checked.so")),
                    reason="checked build not present (python -m minidist._build --bounds-check)")
def test_checked_build_clean_step_matches_normal_build():
    a = _run(_STEP, checked=True)
    b = _run(_STEP, checked=False)
    assert "CHECKED True" in a and "CHECKED False" in b
    la = float(a.split("LOSS ")[1].split()[0])
    lb = float(b.split("LOSS ")[1].split()[0])
    assert abs(la - lb) <= 1e-3 * abs(lb), (la, lb)


@pytest.mark.skipif(not os.path.exists(os.path.join(ROOT, "minidist", "_lib", "libminidist_cuda_checked.so")),
                    reason="checked build not present")
def test_checked_build_reports_a_bad_token_id():
    out = _run(_BAD_ID, checked=True)
    assert "REPORTED" in out and "site 300" in out and "detail 4294967289" in out, out  # -7 as uint32
    out = _run(_BAD_ID, checked=False)
    assert "NOT REPORTED" in out  # the normal build treats it as a row of another shard (zeros)
