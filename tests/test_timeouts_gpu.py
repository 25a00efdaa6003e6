"""Bounded waits in the fused collective kernels, on one GPU, without faulting it.

Each test launches a fused kernel as rank 0 of a two-rank group whose "peer"
buffers are ordinary local allocations that nothing ever writes: the peer's
flags never arrive, the kernel's wait runs out after a short limit (1-2 ms),
records ``kTimeoutPeer`` in the status word and returns.  The host turns that
into ``CommTimeoutError``, and the GPU stays usable: a normal GEMM afterwards
still gives the right answer.
"""

from __future__ import annotations

import ctypes

import pytest
import torch

pytestmark = pytest.mark.gpu


def _after_check():
    from minidist.ops import gemm as G

    x = torch.randn(256, 128, device="cuda").bfloat16()
    w = torch.randn(192, 128, device="cuda").bfloat16()
    y = G.linear_fwd(x, w)
    ref = x.float() @ w.float().t()
    assert ((y.float() - ref).abs().max() / ref.abs().max()).item() < 2e-2


def test_bucket_allreduce_times_out_when_peer_never_arrives():
    from minidist.ops import _native as nat
    from minidist.parallel import collectives as C

    n = 1 << 20
    bufs = [torch.randn(n, device="cuda") for _ in range(2)]
    nflag = int(nat.lib().md_symm_flag_bytes()) // 4
    flags = [torch.zeros(nflag, dtype=torch.int32, device="cuda") for _ in range(2)]
    p = C.ArParams()
    for r in range(2):
        p.bufs[r], p.flags[r] = bufs[r].data_ptr(), flags[r].data_ptr()
    p.offset, p.n, p.world, p.rank, p.scale, p.channel = 0, n, 2, 0, 0.5, 0
    p.timeout_ns = 2_000_000
    p.status = nat.status_ptr()
    nat.check(nat.lib().md_allreduce(ctypes.byref(p), 4, ctypes.c_void_p(nat.stream_ptr())), "md_allreduce")
    with pytest.raises(nat.CommTimeoutError):
        nat.check_status()
    nat.check_status()  # the word was reset
    # The claim counters of channel 0 were reset by the launch's last CTA and the
    # launch was counted (the words behind the flag slots: 3 per channel).
    base = flags[0].numel() - 24
    assert flags[0][base:base + 3].tolist() == [0, 0, 1]
    _after_check()


def test_fused_gemm_allreduce_times_out_when_peer_never_publishes():
    from minidist.ops import _native as nat
    from minidist.ops import gemm as G
    from minidist.parallel import collectives as C

    M, K, N = 512, 128, 512
    x = torch.randn(M, K, device="cuda").bfloat16()
    w = torch.randn(N, K, device="cuda").bfloat16()
    part = [torch.empty(M, N, dtype=torch.bfloat16, device="cuda") for _ in range(2)]
    fin = [torch.empty(M, N, dtype=torch.bfloat16, device="cuda") for _ in range(2)]
    chunks = (M // 32) * ((N + 255) // 256)
    flags = [torch.zeros(2 * chunks, dtype=torch.int32, device="cuda") for _ in range(2)]
    out = torch.empty(M, N, dtype=torch.bfloat16, device="cuda")
    ar = C.TpArParams()
    for r in range(2):
        ar.partial[r], ar.fin[r], ar.flags[r] = part[r].data_ptr(), fin[r].data_ptr(), flags[r].data_ptr()
    ar.ldp, ar.out, ar.ldo = N, out.data_ptr(), N
    ar.world, ar.rank, ar.max_chunks = 2, 0, chunks
    ar.timeout_ns = 1_000_000
    claim = torch.zeros(3, dtype=torch.int32, device="cuda")
    ar.claim = claim.data_ptr()
    gp = nat.GemmParams()
    gp.A, gp.B, gp.lda, gp.ldb = x.data_ptr(), w.data_ptr(), K, K
    gp.M, gp.N, gp.K, gp.epi, gp.alpha = M, N, K, G.EPI_BF16, 1.0
    gp.status = nat.status_ptr()
    rc = nat.lib().md_gemm_ar(ctypes.byref(gp), ctypes.byref(ar), ctypes.c_void_p(nat.stream_ptr()))
    nat.check(rc, "md_gemm_ar")
    with pytest.raises(nat.CommTimeoutError):
        nat.check_status()
    nat.check_status()
    assert claim.tolist() == [0, 0, 1], "cluster-order counters not reset / launch not counted"
    _after_check()
