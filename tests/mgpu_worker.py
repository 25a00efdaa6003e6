"""Worker for tests/test_multigpu_gpu.py (run under torchrun, one process per GPU)."""

from __future__ import annotations

import os
import sys
from datetime import timedelta

import torch
import torch.distributed as dist

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))

from minidist.ops import _native as nat  # noqa: E402
from minidist.parallel import collectives, symm  # noqa: E402


def check_allreduce(rank, world):
    c = symm.communicator(None, list(range(world)))
    assert c is not None, "peer memory unavailable"
    n = 3 * 1024 * 1024 + 64
    buf = symm.SymmBuffer(None, n * 4)
    t = buf.view(torch.float32, 0, n)
    for it in range(3):
        g = torch.Generator(device="cuda").manual_seed(100 + it)
        parts = [torch.randn(n, device="cuda", generator=g) for _ in range(world)]
        t.copy_(parts[rank])
        torch.cuda.synchronize()
        collectives.allreduce_fp32_(buf, c, 0, n, 1.0 / world, 1)
        torch.cuda.synchronize()
        want = torch.stack(parts).sum(0) / world
        err = (t - want).abs().max().item()
        assert err < 1e-5, f"rank {rank} iter {it}: err {err}"
        # every rank holds the identical result
        allv = [torch.empty_like(t) for _ in range(world)]
        dist.all_gather(allv, t)
        assert all(torch.equal(allv[0], a) for a in allv)
    nat.check_status()


def check_ddp(rank, world):
    import minidist as md
    from minidist.models import GPT, GPTConfig
    from minidist.optim import FusedAdamW

    cfg = GPTConfig(vocab_size=1000, block_size=128, n_layer=2, n_head=4, n_embd=256)
    mesh = md.ParallelMesh(tp_size=1)  # data parallel: each rank holds the whole model
    ref = GPT(cfg, tp_group=mesh.tp_group, device="cuda")
    model = md.DistributedDataParallel(GPT(cfg, tp_group=mesh.tp_group, device="cuda"),
                                       process_group=mesh.dp_group, bucket_cap_mb=1.0)
    assert model.reducer_name == "fused-nvlink", model.reducer_name
    g = torch.Generator().manual_seed(7)
    ids = torch.randint(0, cfg.vocab_size, (2 * world, 128), generator=g).cuda()
    tgt = torch.randint(0, cfg.vocab_size, (2 * world, 128), generator=g).cuda()
    with torch.autocast("cuda", dtype=torch.bfloat16):
        ref(ids, tgt)[1].backward()
        model(ids.chunk(world)[rank], tgt.chunk(world)[rank])[1].backward()
    torch.cuda.synchronize()
    for (n, p), (_, q) in zip(model.module.named_parameters(), ref.named_parameters()):
        err = ((p.grad - q.grad).abs().max() / q.grad.abs().max().clamp(min=1e-8)).item()
        assert err < 5e-2, f"rank {rank} {n}: {err}"
    opt = FusedAdamW(model.parameters(), lr=1e-3)
    for _ in range(3):
        opt.zero_grad(set_to_none=True)
        with torch.autocast("cuda", dtype=torch.bfloat16):
            model(ids.chunk(world)[rank], tgt.chunk(world)[rank])[1].backward()
        opt.step()
    torch.cuda.synchronize()
    w = model.module.blocks[0].attn.qkv.weight.detach()
    allw = [torch.empty_like(w) for _ in range(world)]
    dist.all_gather(allw, w)
    assert all(torch.equal(allw[0], a) for a in allw), "replicas diverged"
    nat.check_status()


def main():
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    torch.cuda.set_device(int(os.environ["LOCAL_RANK"]))
    dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=torch.device("cuda", rank))
    try:
        check_allreduce(rank, world)
        check_ddp(rank, world)
    finally:
        symm.release_all()
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
