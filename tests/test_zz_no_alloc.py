"""The allocation-free column-sum entry point (csrc/md_noalloc.h) against md_colsum.

``md_colsum_noalloc`` serves callers that cannot allocate device memory
themselves: its scratch is a static device array inside the library.  This
test calls it through its exported C symbol with ctypes (not through the
Python wrappers), twice in a row on different inputs, and compares each result
with the existing allocating entry point within the tolerance the kernel tests
use.  It also checks that a job needing more scratch than the array holds is
rejected.  The file name sorts last so a ``-x`` run reaches it after every
other test.
"""

from __future__ import annotations

import ctypes

import pytest
import torch

from minidist.ops import _native as nat
from minidist.ops import kernels as K

pytestmark = pytest.mark.gpu

TOO_LARGE = -100  # MD_NOALLOC_TOO_LARGE


def _entry():
    lib = ctypes.CDLL(str(nat.library_path()))
    fn = lib.md_colsum_noalloc
    fn.argtypes = [ctypes.c_void_p, ctypes.c_longlong, ctypes.c_int, ctypes.c_int, ctypes.c_void_p, ctypes.c_int,
                   ctypes.c_void_p]
    fn.restype = ctypes.c_int
    return fn


def _rel(a, b):
    return ((a - b).abs().max() / b.abs().max().clamp(min=1e-6)).item()


def test_noalloc_colsum_matches_allocating_entry_point():
    fn = _entry()
    torch.manual_seed(0)
    stream = torch.cuda.current_stream().cuda_stream
    # Two contiguous shapes (the 8-column vector path), then ragged ones that take the scalar
    # path: N % 8 != 0, and a strided view whose row stride is not a multiple of 8.
    wide = torch.randn(333, 778, device="cuda").bfloat16()  # row stride 778: even, not a multiple of 8
    shapes = [(16384, 3072, False, None), (1000, 768, True, None), (999, 770, False, None),
              (333, 771, True, wide[:, :771])]
    for M, N, accumulate, view in shapes:  # calls in a row, different sizes
        x = torch.randn(M, N, device="cuda").bfloat16() if view is None else view
        base = torch.randn(N, device="cuda")
        want = base.clone()
        K.colsum(x, want, accumulate=accumulate)
        got = base.clone()
        rc = fn(x.data_ptr(), x.stride(0), M, N, got.data_ptr(), int(accumulate), stream)
        assert rc == 0, rc
        torch.cuda.synchronize()
        assert _rel(got, want) < 1e-5
        assert _rel(got, (base if accumulate else 0) + x.float().sum(0)) < 1e-4


def test_noalloc_scratch_size_query_is_64_bit():
    lib = ctypes.CDLL(str(nat.library_path()))
    q = lib.md_colsum_scratch_floats
    q.argtypes, q.restype = [ctypes.c_int, ctypes.c_int], ctypes.c_longlong
    assert q(16384, 20_000_000) > 2**31  # no int overflow for very wide inputs
    assert q(0, 5) == 0


def test_noalloc_colsum_rejects_oversized_jobs():
    fn = _entry()
    M, N = 64, 2_000_000
    x = torch.zeros(M, N, device="cuda", dtype=torch.bfloat16)
    out = torch.zeros(N, device="cuda")
    rc = fn(x.data_ptr(), x.stride(0), M, N, out.data_ptr(), 0, torch.cuda.current_stream().cuda_stream)
    assert rc == TOO_LARGE
