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
        _report(f"peer_allreduce_fp32_w{world}_iter{it}_abs", err, 1e-5, rank)
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
                                       process_group=mesh.dp_group, bucket_cap_mb=1.0, defer_last_buckets=2)
    assert model.reducer_name == "fused-nvlink", model.reducer_name
    g = torch.Generator().manual_seed(7)
    ids = torch.randint(0, cfg.vocab_size, (2 * world, 128), generator=g).cuda()
    tgt = torch.randint(0, cfg.vocab_size, (2 * world, 128), generator=g).cuda()
    with torch.autocast("cuda", dtype=torch.bfloat16):
        ref(ids, tgt)[1].backward()
        model(ids.chunk(world)[rank], tgt.chunk(world)[rank])[1].backward()
    model.wait_gradients()  # the last bucket is deferred (defer_last_buckets=2)
    torch.cuda.synchronize()
    worst = 0.0
    for (n, p), (_, q) in zip(model.module.named_parameters(), ref.named_parameters()):
        worst = max(worst, ((p.grad - q.grad).abs().max() / q.grad.abs().max().clamp(min=1e-8)).item())
    _report(f"ddp_grads_vs_full_batch_w{world}", worst, 5e-2, rank)
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


def check_fsdp(rank, world):
    """FSDP with the peer-memory reduce-scatter: shard gradients equal the full-batch reference's
    shard; the in-kernel AdamW (fused_adamw) matches FSDP + FusedAdamW step for step."""
    import minidist as md
    from minidist.models import GPT, Block, GPTConfig
    from minidist.optim import FusedAdamW

    cfg = GPTConfig(vocab_size=1000, block_size=128, n_layer=2, n_head=4, n_embd=256)
    mesh = md.ParallelMesh(tp_size=1)
    ref = GPT(cfg, tp_group=mesh.tp_group, device="cuda")
    model = md.FullyShardedDataParallel(GPT(cfg, tp_group=mesh.tp_group, device="cuda"), unit_types=(Block,),
                                        process_group=mesh.dp_group)
    assert all(u._peer is not None for u in model._units), "peer-memory reduce-scatter not in use"
    assert all(u._peer_shard is not None for u in model._units), "peer-memory gather not in use"
    # bf16 gather (md_ag_shards): the gathered unit is exactly every rank's fp32 shard cast to bf16.
    mp = md.FullyShardedDataParallel(GPT(cfg, tp_group=mesh.tp_group, device="cuda"), unit_types=(Block,),
                                     process_group=mesh.dp_group,
                                     mixed_precision=md.MixedPrecisionPolicy(param_dtype=torch.bfloat16))
    for u in mp._units:
        with torch.no_grad():
            u.flat_shard.add_(torch.randn_like(u.flat_shard) * (rank + 1))  # distinct shards per rank
        u.unshard()
        full = torch.empty(u.padded_numel, dtype=torch.float32, device="cuda")
        dist.all_gather_into_tensor(full, u.flat_shard.detach(), group=mesh.dp_group)
        assert torch.equal(u._full, full.bfloat16()), f"rank {rank} unit {u.name}: bf16 gather differs"
        u.reshard()
    g = torch.Generator().manual_seed(11)
    ids = torch.randint(0, cfg.vocab_size, (2 * world, 128), generator=g).cuda()
    tgt = torch.randint(0, cfg.vocab_size, (2 * world, 128), generator=g).cuda()
    with torch.autocast("cuda", dtype=torch.bfloat16):
        ref(ids, tgt)[1].backward()
        model(ids.chunk(world)[rank], tgt.chunk(world)[rank])[1].backward()
    model.finish_gradient_sync()
    torch.cuda.synchronize()
    refp = dict(ref.named_parameters())
    names = {id(p): n for n, p in model.module.named_parameters()}
    for u in model._units:
        full = torch.cat([refp[names[id(p)]].grad.reshape(-1).float() for p in u.params])
        full = torch.cat([full, full.new_zeros(u.padded_numel - u.total_numel)])
        want = full[rank * u.shard_numel:(rank + 1) * u.shard_numel]
        err = ((u.flat_shard.grad - want).abs().max() / want.abs().max().clamp(min=1e-8)).item()
        _report(f"fsdp_shard_grad_w{world}_unit_{u.name}", err, 5e-2, rank)
    # in-kernel AdamW vs FusedAdamW on the same FSDP shards
    hp = dict(lr=1e-3, betas=(0.9, 0.999), eps=1e-8, weight_decay=0.01)
    fa = md.FullyShardedDataParallel(GPT(cfg, tp_group=mesh.tp_group, device="cuda"), unit_types=(Block,),
                                     process_group=mesh.dp_group, fused_adamw=hp)
    fb = md.FullyShardedDataParallel(GPT(cfg, tp_group=mesh.tp_group, device="cuda"), unit_types=(Block,),
                                     process_group=mesh.dp_group)
    opt = FusedAdamW(fb.parameters(), **hp)
    for it in range(3):
        x = ids.roll(it, 1).chunk(world)[rank]
        y = tgt.roll(it, 1).chunk(world)[rank]
        with torch.autocast("cuda", dtype=torch.bfloat16):
            fa(x, y)[1].backward()
        fa.finish_gradient_sync()
        opt.zero_grad(set_to_none=True)
        with torch.autocast("cuda", dtype=torch.bfloat16):
            fb(x, y)[1].backward()
        fb.finish_gradient_sync()
        opt.step()
    torch.cuda.synchronize()
    for ua, ub in zip(fa._units, fb._units):
        assert ua.flat_shard.grad is None, "fused AdamW left a shard gradient behind"
        d = (ua.flat_shard.data - ub.flat_shard.data).abs().max().item()
        _report(f"fsdp_inkernel_adamw_w{world}_unit_{ua.name}_abs", d, 1e-4, rank)
    nat.check_status()


def check_gemm_ar(rank, world):
    """Fused GEMM + all-reduce (md_gemm_ar) against fp32 torch on the gathered partials."""
    for it, (M, K, N, with_resid) in enumerate([(1000, 192, 768, True), (4096, 384, 768, False),
                                                (333, 64, 200, True), (4096, 96, 768, True)]):
        g = torch.Generator(device="cuda").manual_seed(10 + it)
        xs = [torch.randn(M, K, device="cuda", generator=g).bfloat16() for _ in range(world)]
        ws = [(torch.randn(N, K, device="cuda", generator=g) * 0.05).bfloat16() for _ in range(world)]
        bias = torch.randn(N, device="cuda", generator=g)
        resid = torch.randn(M, N, device="cuda", generator=g).bfloat16() if with_resid else None
        out = collectives.gemm_all_reduce(xs[rank], ws[rank], bias, resid, None)
        torch.cuda.synchronize()
        want = sum(x.float() @ w.float().t() for x, w in zip(xs, ws)) + bias
        if resid is not None:
            want = want + resid.float()
        err = ((out.float() - want).abs().max() / want.abs().max()).item()
        _report(f"gemm_allreduce_w{world}_case{it}_M{M}_K{K}_N{N}", err, 2e-2, rank)
        allo = [torch.empty(M, N, dtype=torch.bfloat16, device="cuda") for _ in range(world)]
        dist.all_gather(allo, out.contiguous())
        assert all(torch.equal(allo[0], a) for a in allo), f"case {it}: ranks differ"
    nat.check_status()


def check_tp_gpt(rank, world):
    """GPT with tensor parallelism over every rank (fused row-parallel GEMM + all-reduce) vs tp=1."""
    import minidist as md
    from minidist.models import GPT, GPTConfig

    cfg = GPTConfig(vocab_size=1024, block_size=128, n_layer=2, n_head=8, n_embd=512)
    mesh = md.ParallelMesh(tp_size=world)
    solo = md.ParallelMesh(tp_size=1)
    ref = GPT(cfg, tp_group=solo.tp_group, device="cuda")
    model = GPT(cfg, tp_group=mesh.tp_group, device="cuda")
    g = torch.Generator().manual_seed(3)
    ids = torch.randint(0, cfg.vocab_size, (4, 128), generator=g).cuda()
    tgt = torch.randint(0, cfg.vocab_size, (4, 128), generator=g).cuda()
    with torch.autocast("cuda", dtype=torch.bfloat16):
        l_ref = ref(ids, tgt)[1]
        l_tp = model(ids, tgt)[1]
    l_ref.backward()
    l_tp.backward()
    torch.cuda.synchronize()
    _report(f"tp_gpt_w{world}_loss", abs(l_ref.item() - l_tp.item()) / abs(l_ref.item()), 2e-2, rank)
    # the row-parallel weight gradient is this rank's column slice of the full gradient
    gfull = ref.blocks[0].mlp.proj.weight.grad
    gpart = model.blocks[0].mlp.proj.weight.grad
    cols = gpart.shape[1]
    want = gfull[:, rank * cols:(rank + 1) * cols]
    err = ((gpart - want).abs().max() / want.abs().max()).item()
    _report(f"tp_gpt_w{world}_mlp_proj_grad", err, 5e-2, rank)
    # position-embedding gradient: downstream of every fused data-gradient all-reduce
    gw, gr = model.embedding.wpe.grad, ref.embedding.wpe.grad
    err = ((gw - gr).abs().max() / gr.abs().max()).item()
    _report(f"tp_gpt_w{world}_wpe_grad", err, 5e-2, rank)
    nat.check_status()


def _graph_vs_eager(rank, world, wrap, tp_size):
    """Train the same model eagerly and as a replayed CUDA graph (GraphedStep); losses must agree."""
    import minidist as md
    from minidist.models import GPT, GPTConfig
    from minidist.optim import FusedAdamW

    cfg = GPTConfig(vocab_size=1024, block_size=128, n_layer=2, n_head=4, n_embd=256, seed=9)
    g = torch.Generator().manual_seed(21)
    batches = [(torch.randint(0, cfg.vocab_size, (2, 128), generator=g).cuda(),
                torch.randint(0, cfg.vocab_size, (2, 128), generator=g).cuda()) for _ in range(6)]
    out = []
    for graph in (False, True):
        mesh = md.ParallelMesh(tp_size=tp_size)
        model = wrap(GPT(cfg, tp_group=mesh.tp_group, device="cuda"), mesh)
        opt = FusedAdamW(model.parameters(), lr=1e-3, capturable=graph)

        def step(x, y):
            opt.zero_grad(set_to_none=True)
            with torch.autocast("cuda", dtype=torch.bfloat16, cache_enabled=False):
                loss = model(x, y)[1]
            loss.backward()
            opt.step()
            return loss

        if graph:
            run = md.GraphedStep(step, batches[0], warmup=2, optimizers=[opt])
        else:
            step(*batches[0])
            step(*batches[0])
            run = step
        losses = [float(run(*b).item()) for b in batches[1:]]
        if graph:
            run.release()
        out.append(losses)
    _report(f"cuda_graph_vs_eager_w{world}_tp{tp_size}_losses",
            max(abs(a - b) / abs(a) for a, b in zip(*out, strict=True)), 3e-3, rank)
    nat.check_status()


def check_graphs(rank, world):
    """DDP (peer-memory bucket all-reduce) and tensor parallelism (fused GEMM + all-reduce) inside
    a CUDA graph: the device-counted barrier epochs keep replays correct."""
    import minidist as md

    _graph_vs_eager(rank, world, lambda m, mesh: md.DistributedDataParallel(
        m, process_group=mesh.dp_group, bucket_cap_mb=1.0, defer_last_buckets=2), tp_size=1)
    _graph_vs_eager(rank, world, lambda m, mesh: m, tp_size=world)


def _rel(a, b) -> float:
    return ((a.float() - b.float()).abs().max() / b.float().abs().max().clamp(min=1e-8)).item()


def _report(name: str, err: float, tol: float, rank: int) -> None:
    """One line per check for the summary table (rank 0), then the assertion."""
    if rank == 0:
        print(f"CHECK {name} max_rel_err={err:.3e} tol={tol:.0e} {'PASS' if err < tol else 'FAIL'}", flush=True)
    assert err < tol, f"rank {rank} {name}: {err} >= {tol}"


def _stage_model(cfg, mesh):
    """This pipeline stage's slice of the GPT layers, with the fused LM-head loss on the last stage."""
    import minidist as md
    from torch import nn

    from minidist.models import build_pipeline_layers

    layers = build_pipeline_layers(cfg, tp_group=mesh.tp_group, device="cuda")
    mine = md.partition_layers(layers, mesh.pp_size, mesh.pp_rank)
    loss_fn = None
    if mesh.is_last_stage:
        head = mine[-1]
        head.loss_only = True

        def loss_fn(hidden, targets):
            return head.loss(hidden, targets)
    return nn.Sequential(*mine), loss_fn, len(layers)


def _stage_param_names(mesh, n_layers):
    """Names in the unwrapped GPT of this stage's parameters, in the order of ``nn.Sequential``."""
    from minidist.pipeline import partition_layers

    idx = partition_layers(list(range(n_layers)), mesh.pp_size, mesh.pp_rank)
    names = []
    for i in idx:
        prefix = "embedding" if i == 0 else ("lm_head" if i == n_layers - 1 else f"blocks.{i - 1}")
        names.append(prefix)
    return idx, names


def check_pipeline(rank, world):
    """GPipe and 1F1B over ``world`` stages (NCCL send / recv, fused blocks) reproduce the single-stage
    loss and every stage's parameter gradients (reference tests/test_pipeline.py:53-97)."""
    import minidist as md
    from minidist.models import GPT, GPTConfig

    cfg = GPTConfig(vocab_size=1024, block_size=128, n_layer=2 * world, n_head=4, n_embd=256, seed=5)
    g = torch.Generator().manual_seed(17)
    ids = torch.randint(0, cfg.vocab_size, (8, 128), generator=g).cuda()
    tgt = torch.randint(0, cfg.vocab_size, (8, 128), generator=g).cuda()
    solo = md.ParallelMesh(tp_size=1, pp_size=1, dp_size=world)
    ref = GPT(cfg, tp_group=solo.tp_group, device="cuda")
    with torch.autocast("cuda", dtype=torch.bfloat16):
        l_ref = ref(ids, tgt)[1]
    l_ref.backward()
    refp = dict(ref.named_parameters())
    mesh = md.ParallelMesh(tp_size=1, pp_size=world)
    for sched in ("gpipe", "1f1b"):
        core, loss_fn, n_layers = _stage_model(cfg, mesh)
        stage = md.PipelineStage(core, mesh, loss_fn=loss_fn)
        schedule = md.build_schedule(sched, stage, mesh, 4)
        with torch.autocast("cuda", dtype=torch.bfloat16):
            loss = schedule.step(inputs=ids, targets=tgt)
        torch.cuda.synchronize()
        v = torch.zeros(1, device="cuda")
        if loss is not None:
            v[0] = loss
        dist.broadcast(v, src=mesh.pp_ranks[-1], group=mesh.pp_group)
        _report(f"pipeline_{sched}_w{world}_loss", abs(v.item() - l_ref.item()) / abs(l_ref.item()), 2e-2, rank)
        worst = 0.0
        _, prefixes = _stage_param_names(mesh, n_layers)
        for mod, prefix in zip(core, prefixes):
            for n, p in mod.named_parameters():
                worst = max(worst, _rel(p.grad, refp[f"{prefix}.{n}"].grad))
        _report(f"pipeline_{sched}_w{world}_grads", worst, 6e-2, rank)
        if sched == "1f1b" and world > 1:
            assert schedule.max_activations_in_flight <= world - mesh.pp_rank
    nat.check_status()


def check_composition(rank, world):
    """tp2 x pp2 x dp(world/4): 1F1B with 4 microbatches per replica and DDP over the data-parallel
    group vs the single-process full batch (reference tests/test_composition.py:62-157)."""
    import minidist as md
    from minidist.models import GPT, GPTConfig

    if world % 4:
        return
    cfg = GPTConfig(vocab_size=1024, block_size=128, n_layer=4, n_head=8, n_embd=512, seed=6)
    dp = world // 4
    g = torch.Generator().manual_seed(23)
    ids = torch.randint(0, cfg.vocab_size, (4 * dp, 128), generator=g).cuda()
    tgt = torch.randint(0, cfg.vocab_size, (4 * dp, 128), generator=g).cuda()
    solo = md.ParallelMesh(tp_size=1, pp_size=1, dp_size=world)
    ref = GPT(cfg, tp_group=solo.tp_group, device="cuda")
    with torch.autocast("cuda", dtype=torch.bfloat16):
        l_ref = ref(ids, tgt)[1]
    l_ref.backward()
    refp = dict(ref.named_parameters())
    mesh = md.ParallelMesh(tp_size=2, pp_size=2)
    core, loss_fn, n_layers = _stage_model(cfg, mesh)
    model = md.DistributedDataParallel(core, process_group=mesh.dp_group, bucket_cap_mb=1.0) if dp > 1 else core
    stage = md.PipelineStage(model, mesh, loss_fn=loss_fn)
    schedule = md.build_schedule("1f1b", stage, mesh, 4)
    mine = slice(mesh.dp_rank * 4, (mesh.dp_rank + 1) * 4)
    ctx = model.no_sync() if dp > 1 else torch.enable_grad()
    with ctx, torch.autocast("cuda", dtype=torch.bfloat16):
        loss = schedule.step(inputs=ids[mine], targets=tgt[mine])
    if dp > 1:
        model.finish_gradient_sync()
    torch.cuda.synchronize()
    v = torch.zeros(1, device="cuda")
    if loss is not None:
        v[0] = loss
    dist.all_reduce(v, group=mesh.pp_group)  # only the last stage holds it
    dist.all_reduce(v, group=mesh.dp_group)
    v /= mesh.dp_size
    _report(f"composition_tp2pp2dp{dp}_loss", abs(v.item() - l_ref.item()) / abs(l_ref.item()), 2e-2, rank)
    # Every parameter's gradient is this rank's tensor-parallel slice of the reference gradient.
    worst = 0.0
    _, prefixes = _stage_param_names(mesh, n_layers)
    for mod, prefix in zip(core, prefixes):
        for n, p in mod.named_parameters():
            full = refp[f"{prefix}.{n}"].grad
            if p.shape != full.shape:
                dim = next(d for d in range(p.dim()) if p.shape[d] != full.shape[d])
                full = full.chunk(mesh.tp_size, dim=dim)[mesh.tp_rank]
            worst = max(worst, _rel(p.grad, full))
    _report(f"composition_tp2pp2dp{dp}_grads", worst, 6e-2, rank)
    nat.check_status()


def check_fsdp_training(rank, world):
    """Four AdamW steps of FSDP, with bf16 and with fp32 parameter gathers, track DDP's weights
    (reference tests/test_fsdp.py:92-127, 189-211)."""
    for pdt in (torch.bfloat16, torch.float32):
        _fsdp_training(rank, world, pdt)


def _fsdp_training(rank, world, param_dtype):
    import minidist as md
    from minidist.models import GPT, Block, GPTConfig
    from minidist.optim import FusedAdamW

    tag = "bf16" if param_dtype == torch.bfloat16 else "fp32"
    cfg = GPTConfig(vocab_size=1024, block_size=128, n_layer=2, n_head=4, n_embd=256, seed=8)
    mesh = md.ParallelMesh(tp_size=1)
    ddp = md.DistributedDataParallel(GPT(cfg, tp_group=mesh.tp_group, device="cuda"), process_group=mesh.dp_group)
    fsdp = md.FullyShardedDataParallel(GPT(cfg, tp_group=mesh.tp_group, device="cuda"), unit_types=(Block,),
                                       process_group=mesh.dp_group,
                                       mixed_precision=md.MixedPrecisionPolicy(param_dtype=param_dtype))
    o1 = FusedAdamW(ddp.parameters(), lr=1e-3)
    o2 = FusedAdamW(fsdp.parameters(), lr=1e-3)
    g = torch.Generator().manual_seed(31)
    losses = []
    for it in range(4):
        ids = torch.randint(0, cfg.vocab_size, (2, 128), generator=g).cuda()
        tgt = torch.randint(0, cfg.vocab_size, (2, 128), generator=g).cuda()
        pair = []
        for model, opt in ((ddp, o1), (fsdp, o2)):
            opt.zero_grad(set_to_none=True)
            with torch.autocast("cuda", dtype=torch.bfloat16):
                loss = model(ids, tgt)[1]
            loss.backward()
            opt.step()
            pair.append(loss.item())
        losses.append(pair)
    torch.cuda.synchronize()
    # The losses see the forward weights directly: stale gathered weights (or stale casts of
    # them) show up here at the 1e-2 level after four steps, reduction-order noise at 1e-4.
    _report(f"fsdp_{tag}_vs_ddp_w{world}_losses", max(abs(a - b) / abs(a) for a, b in losses), 2e-3, rank)
    worst = 0.0
    with fsdp.summon_full_params():
        for (n, p), (_, q) in zip(fsdp.module.named_parameters(), ddp.module.named_parameters()):
            worst = max(worst, (p.float() - q.float()).abs().max().item())
    # Adam turns reduction-order differences of tiny gradients into steps of up to ~lr each.
    _report(f"fsdp_{tag}_vs_ddp_w{world}_weights_abs", worst, 2e-2, rank)
    nat.check_status()


def check_tp_embedding(rank, world):
    """md_embed_tp: each row read from its owner's bf16 shard equals the masked-lookup + all-reduce."""
    import minidist as md
    from minidist.models import GPT, GPTConfig

    cfg = GPTConfig(vocab_size=1024 * world, block_size=128, n_layer=1, n_head=8, n_embd=512, seed=4)
    mesh = md.ParallelMesh(tp_size=world)
    model = GPT(cfg, tp_group=mesh.tp_group, device="cuda")
    g = torch.Generator().manual_seed(3)
    ids = torch.randint(0, cfg.vocab_size, (4, 128), generator=g).cuda()
    with torch.autocast("cuda", dtype=torch.bfloat16):
        x = model.embedding(ids)
    emb = model.embedding
    full = torch.empty(cfg.vocab_size, cfg.n_embd, device="cuda")
    dist.all_gather_into_tensor(full, emb.wte.weight.detach(), group=mesh.tp_group)
    want = (full.bfloat16().float()[ids] + emb.wpe.detach().bfloat16().float()[:128]).bfloat16()
    _report(f"tp_embedding_w{world}", _rel(x, want), 1e-2, rank)
    allx = [torch.empty_like(x) for _ in range(world)]
    dist.all_gather(allx, x.contiguous())
    assert all(torch.equal(allx[0], a) for a in allx), "embedding differs across TP ranks"
    nat.check_status()


def main():
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    torch.cuda.set_device(int(os.environ["LOCAL_RANK"]))
    dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=torch.device("cuda", rank))
    checks = {"allreduce": check_allreduce, "gemm_ar": check_gemm_ar, "ddp": check_ddp, "fsdp": check_fsdp,
              "tp_gpt": check_tp_gpt, "tp_embedding": check_tp_embedding, "graphs": check_graphs,
              "pipeline": check_pipeline, "composition": check_composition, "fsdp_training": check_fsdp_training}
    # MGPU_CHECKS=name,name runs a subset (same order); default: all of them.
    wanted = [c for c in os.environ.get("MGPU_CHECKS", "").split(",") if c] or list(checks)
    unknown = [c for c in wanted if c not in checks]
    if unknown:
        raise SystemExit(f"unknown checks {unknown}; known: {list(checks)}")
    try:
        for name in checks:
            if name in wanted:
                checks[name](rank, world)
    finally:
        symm.release_all()
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
