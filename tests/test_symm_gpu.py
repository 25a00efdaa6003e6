"""The peer-memory collective kernels (csrc/symm.cu) as a group of one rank, on one GPU.

Every "peer" pointer is this rank's own buffer, so these check the kernels'
indexing, casts and counters against fp32 PyTorch; the multi-rank behaviour is
covered by tests/test_multigpu_gpu.py.
"""

from __future__ import annotations

import ctypes

import pytest
import torch

pytestmark = pytest.mark.gpu


def _flags():
    from minidist.ops import _native as nat

    return torch.zeros(int(nat.lib().md_symm_flag_bytes()) // 4, dtype=torch.int32, device="cuda")


def _counters(flags, channel):
    """(claimed, finished, launches) of ``channel``: the three words per channel behind the flag slots."""
    base = flags.numel() - 3 * 8 + 3 * channel
    return flags[base:base + 3].tolist()


@pytest.mark.parametrize("out_dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("shard,offset", [(4096, 0), (1 << 20, 12), (40_000, 100)])
def test_all_gather_shards_world1(out_dtype, shard, offset):
    from minidist.ops import _native as nat
    from minidist.parallel import collectives as C

    buf = torch.randn(offset + shard + 64, device="cuda")
    flags = _flags()
    out = torch.full((shard,), 7.0, device="cuda").to(out_dtype)
    p = C.AgParams()
    p.bufs[0], p.flags[0] = buf.data_ptr(), flags.data_ptr()
    p.offset, p.shard, p.world, p.rank, p.channel = offset, shard, 1, 0, 5
    p.timeout_ns, p.status = 10**10, nat.status_ptr()
    p.out, p.out_bf16 = out.data_ptr(), int(out_dtype == torch.bfloat16)
    for _ in range(2):
        ctas = min(64, max(1, shard // 65536))
        nat.check(nat.lib().md_ag_shards(ctypes.byref(p), ctas, ctypes.c_void_p(nat.stream_ptr())), "md_ag_shards")
    nat.check_status()
    assert torch.equal(out, buf[offset:offset + shard].to(out_dtype))
    assert _counters(flags, 5) == [0, 0, 2], "claim counters not reset / launches not counted"


def test_reduce_scatter_shard_adamw_world1():
    from minidist.ops import _native as nat
    from minidist.parallel import collectives as C

    shard = 3 * 65536 + 4
    g = torch.randn(shard, device="cuda")
    p0, m0, v0 = torch.randn(shard, device="cuda"), torch.randn(shard, device="cuda") * 0.1, torch.rand(shard, device="cuda")
    p, m, v = p0.clone(), m0.clone(), v0.clone()
    flags = _flags()
    r = C.RsParams()
    r.bufs[0], r.flags[0] = g.data_ptr(), flags.data_ptr()
    r.offset, r.shard, r.world, r.rank, r.scale, r.channel = 0, shard, 1, 0, 0.5, 4
    r.timeout_ns, r.status = 10**10, nat.status_ptr()
    r.p, r.m, r.v = p.data_ptr(), m.data_ptr(), v.data_ptr()
    lr, b1, b2, eps, wd, step = 1e-3, 0.9, 0.999, 1e-8, 0.01, 3
    r.lr, r.b1, r.b2, r.eps, r.wd = lr, b1, b2, eps, wd
    r.bc1, r.bc2_sqrt = 1 - b1 ** step, (1 - b2 ** step) ** 0.5
    nat.check(nat.lib().md_rs_shard(ctypes.byref(r), 37, ctypes.c_void_p(nat.stream_ptr())), "md_rs_shard")
    nat.check_status()
    gs = g * 0.5
    m_ref = b1 * m0 + (1 - b1) * gs
    v_ref = b2 * v0 + (1 - b2) * gs * gs
    p_ref = p0 * (1 - lr * wd) - lr / r.bc1 * m_ref / (v_ref.sqrt() / r.bc2_sqrt + eps)
    torch.testing.assert_close(m, m_ref, rtol=1e-5, atol=1e-6)
    torch.testing.assert_close(v, v_ref, rtol=1e-5, atol=1e-6)
    torch.testing.assert_close(p, p_ref, rtol=1e-5, atol=1e-5)
    assert _counters(flags, 4) == [0, 0, 1]


def test_bucket_allreduce_world1_scale():
    from minidist.ops import _native as nat
    from minidist.parallel import collectives as C

    n = 5 * 65536 + 8
    buf = torch.randn(n + 16, device="cuda")
    want = buf.clone()
    want[16:] *= 0.25
    flags = _flags()
    p = C.ArParams()
    p.bufs[0], p.flags[0] = buf.data_ptr(), flags.data_ptr()
    p.offset, p.n, p.world, p.rank, p.scale, p.channel = 16, n, 1, 0, 0.25, 0
    p.timeout_ns, p.status = 10**10, nat.status_ptr()
    ctas = nat.lib().md_allreduce_ctas(n, 1)
    nat.check(nat.lib().md_allreduce(ctypes.byref(p), ctas, ctypes.c_void_p(nat.stream_ptr())), "md_allreduce")
    nat.check_status()
    torch.testing.assert_close(buf, want, rtol=0, atol=0)
    assert _counters(flags, 0) == [0, 0, 1]


def test_ce_tp_stats_world1():
    """md_ce_tp as a group of one equals the single-GPU statistics kernel (lse and per-row loss)."""
    from minidist.ops import _native as nat
    from minidist.ops import kernels as K
    from minidist.parallel import collectives as C

    tiles, M = 7, 3000
    tmax = torch.randn(tiles, M, device="cuda") * 3
    tmax[2, :100] = float("-inf")  # empty slabs are skipped
    tsum = torch.rand(tiles, M, device="cuda") * 50 + 1
    ttgt = torch.randn(M, device="cuda")
    buf = torch.zeros(3 * M, device="cuda")
    flags = _flags()
    lse, loss = torch.empty(M, device="cuda"), torch.empty(M, device="cuda")
    p = C.CeTpParams()
    p.bufs[0], p.flags[0] = buf.data_ptr(), flags.data_ptr()
    p.world, p.rank, p.channel, p.timeout_ns, p.status = 1, 0, 6, 10**10, nat.status_ptr()
    p.tmax, p.tsum, p.tiles, p.ttgt, p.M = tmax.data_ptr(), tsum.data_ptr(), tiles, ttgt.data_ptr(), M
    p.lse, p.loss = lse.data_ptr(), loss.data_ptr()
    nat.check(nat.lib().md_ce_tp(ctypes.byref(p), 12, ctypes.c_void_p(nat.stream_ptr())), "md_ce_tp")
    nat.check_status()
    _, _, want_lse, want_loss = K.ce_stats(tmax, tsum, ttgt, finish=True)
    torch.testing.assert_close(lse, want_lse, rtol=1e-5, atol=1e-5)
    torch.testing.assert_close(loss, want_loss, rtol=1e-5, atol=1e-5)
    assert _counters(flags, 6) == [0, 0, 1]
