#!/usr/bin/env python3
"""Headline benchmark: GPT training throughput (tokens/s for the whole job), both frameworks.

Configurations (BASELINE.json's five; ``--config``, default ``gpt2s-ddp``):

  gpt2s-ddp     GPT-2 small 12L/768d/12h, vocab 50257, seq 1024, 16 seqs/GPU, DDP with 25 MB
                buckets overlapped with backward (weak scaling: dp = N)
  gpt1.5b-fsdp  GPT 1.5B 48L/1600d/25h, vocab 50257, seq 1024, 8 seqs/GPU, ZeRO-3 with bf16
                parameter gathers, fp32 master weights and fp32 gradient reduce-scatter, one
                unit per block (weak scaling: dp = N; N = 1 trains the unwrapped model)
  gpt2.7b-3d    GPT 2.7B 32L/2560d/32h, vocab 50304, seq 2048, tp2 x pp2 x dp(N/4), 1F1B with
                8 microbatches (``--schedule gpipe`` for the secondary run), 32 seqs per
                data-parallel replica (global batch 64 at N = 8)
  gpt6.7b-tp8   GPT 6.7B 32L/4096d/32h, vocab 50304, seq 2048, 4 seqs, tensor parallel over
                all N GPUs (strong scaling; the named config is N = 8)

Every configuration runs bf16 autocast compute, AdamW (lr 3e-4), synthetic
uniform-random tokens seeded by ``seed + step*10000 + dp_rank`` and random-init
weights of the named architecture.

    python bench.py                                      # 1 GPU, our framework, gpt2s-ddp
    python bench.py --impl reference                     # the unmodified reference (baseline/_ref)
    torchrun --nproc-per-node 8 bench.py --gpus 8 --config gpt6.7b-tp8

Arms.  ``--impl ours`` builds the model through this repository's public API
(GPT on the fused sm_100a path, DistributedDataParallel / FullyShardedDataParallel /
PipelineStage + build_schedule, FusedAdamW).  ``--impl reference`` builds the same
configuration through the reference package's own public API and stock code path
(its GPT, DDP, FSDP, pipeline schedules and vocab-parallel cross-entropy, torch
AdamW, bf16 autocast -- what its examples/train_gpt.py:120-218 does), imported
from ``baseline/_ref``.

Timing: W warm-up steps, then exactly K steps bracketed by a barrier and
torch.cuda.synchronize() on both sides, timed with CUDA events on the compute
stream; the reported step time is the maximum over ranks.  Every step's working
set (activations of several GB plus the weights) is far larger than the 126 MB
L2, so no explicit flush is needed.  SM clocks and throttle reasons are sampled
with nvidia-smi during the timed region.  Our arm replays data-parallel and
tensor-parallel steps as one CUDA graph (minidist.GraphedStep; ``--no-graph``
runs eagerly); FSDP and pipeline steps run eagerly.

The ``e2e`` block repeats the K steps through the same public API with the
inputs copied from pinned host memory each step and the loss read back to the
host each step (wall clock, max over ranks).
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
REF_PATH = os.path.join(ROOT, "baseline", "_ref")

METRIC = "GPT train tokens/s/box at 1/2/4/8 B200 (DDP,FSDP,TP×PP×DP), max over ranks"

# name -> model shape, per-replica batch and parallel layout.
CONFIGS = {
    "gpt2s-ddp": dict(model="gpt2-small 12L/768d/12h, vocab 50257 (untied head)",
                      vocab=50257, layers=12, heads=12, embd=768, seq=1024, batch=16,
                      strategy="ddp", tp=1, pp=1, scaling="weak"),
    "gpt1.5b-fsdp": dict(model="gpt 1.5B 48L/1600d/25h, vocab 50257", vocab=50257, layers=48, heads=25,
                         embd=1600, seq=1024, batch=8, strategy="fsdp", tp=1, pp=1, scaling="weak"),
    "gpt2.7b-3d": dict(model="gpt 2.7B 32L/2560d/32h, vocab 50304", vocab=50304, layers=32, heads=32,
                       embd=2560, seq=2048, batch=32, strategy="ddp", tp=2, pp=2, microbatches=8,
                       scaling="weak"),
    "gpt6.7b-tp8": dict(model="gpt 6.7B 32L/4096d/32h, vocab 50304", vocab=50304, layers=32, heads=32,
                        embd=4096, seq=2048, batch=4, strategy="none", tp=-1, pp=1, scaling="strong"),
}
# Small shapes of the same layouts, for CPU wiring tests (``--tiny``; never a headline number).
_TINY = dict(vocab=256, layers=4, heads=4, embd=64, seq=32)


def parse_args(argv=None):
    p = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=30)
    p.add_argument("--warmup", type=int, default=3)
    p.add_argument("--impl", choices=["ours", "reference"], default="ours")
    p.add_argument("--config", choices=sorted(CONFIGS), default="gpt2s-ddp")
    p.add_argument("--schedule", choices=["1f1b", "gpipe"], default="1f1b", help="pipeline configs only")
    p.add_argument("--seed", type=int, default=1234)
    p.add_argument("--no-e2e", action="store_true")
    p.add_argument("--no-graph", action="store_true", help="our arm: run the step eagerly (no CUDA graph)")
    p.add_argument("--device", choices=["cuda", "cpu"], default="cuda",
                   help="cpu: Gloo wiring check of both arms (host timing; not a benchmark)")
    p.add_argument("--tiny", action="store_true", help="small model of the same layout (wiring checks only)")
    return p.parse_args(argv)


def resolve_config(name: str, world: int, tiny: bool = False) -> dict:
    """The configuration with its layout resolved for ``world`` ranks."""
    c = dict(CONFIGS[name])
    if tiny:
        c.update(_TINY, batch=4, model=c["model"] + " [tiny]")
        if "microbatches" in c:
            c["microbatches"] = 2
    if c["tp"] == -1:
        c["tp"] = world
    if world % (c["tp"] * c["pp"]):
        raise SystemExit(f"--config {name} needs a multiple of tp*pp = {c['tp'] * c['pp']} ranks, got {world}")
    c["dp"] = world // (c["tp"] * c["pp"])
    if c["strategy"] == "none" and c["dp"] > 1:
        raise SystemExit(f"--config {name} has no data-parallel axis; use exactly tp*pp ranks")
    return c


# ---------------------------------------------------------------------------
# Clock sampling (nvidia-smi, read-only)
# ---------------------------------------------------------------------------

_REASONS = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]


class ClockSampler:
    """One ``nvidia-smi -lms 100`` process per node, over every GPU of the run.

    Started before the warm-up steps (its NVML start-up takes host CPU and must
    not overlap the timed window); each sample is stamped on arrival and
    :meth:`stop` keeps the samples inside ``[t0, t1]``, the timed window.
    """

    def __init__(self, gpu_ids: list[str]):
        self.gpu_ids = gpu_ids
        self.rows: list[tuple[float, list[str]]] = []
        self.proc = None
        self.thread = None

    def start(self):
        q = ("clocks.sm,clocks.max.sm,power.draw,utilization.gpu,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={q}", "--format=csv,noheader,nounits", "-lms", "100",
                 "-i", ",".join(self.gpu_ids)],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None
            return
        self.thread = threading.Thread(target=self._read, daemon=True)
        self.thread.start()

    def _read(self):
        for line in self.proc.stdout:
            parts = [x.strip() for x in line.split(",")]
            if len(parts) == 8:
                self.rows.append((time.time(), parts))

    def stop(self, t0: float, t1: float) -> dict:
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        if self.thread is not None:
            self.thread.join(timeout=5)

        def num(s):
            try:
                return float(s)
            except ValueError:
                return None

        # Samples inside the timed window (a sample arrives up to one period after it was taken).
        window = [r for t, r in self.rows if t0 <= t <= t1 + 0.15]
        if not window:  # window shorter than the sampling period: take the samples closest to it
            near = sorted(self.rows, key=lambda tr: abs(tr[0] - (t0 + t1) / 2))
            window = [r for _, r in near[: len(self.gpu_ids)]]
        loaded = [r for r in window if (num(r[3]) or 0) >= 50] or window
        sm = [num(r[0]) for r in loaded if num(r[0]) is not None]
        mx = [num(r[1]) for _, r in self.rows if num(r[1]) is not None]
        reasons = sorted({name for r in loaded for name, v in zip(_REASONS, r[4:8]) if v.lower() == "active"})
        return {
            "sm_mhz": statistics.median(sm) if sm else None,
            "sm_max_mhz": max(mx) if mx else None,
            "reasons": reasons,
            "samples": len(window),
            "gpus": len(self.gpu_ids),
            "power_w_max": max((num(r[2]) or 0) for r in window) if window else None,
        }


# ---------------------------------------------------------------------------
# Distributed setup
# ---------------------------------------------------------------------------


def setup(args):
    import torch
    import torch.distributed as dist
    from datetime import timedelta

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world != args.gpus:
        raise SystemExit(f"--gpus {args.gpus} but WORLD_SIZE={world}; launch N>1 with torchrun")
    os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
    # A short process-group timeout ends a collective that a failed rank never joins.
    pg_timeout = timedelta(seconds=float(os.environ.get("MINIDIST_PG_TIMEOUT_S", "600")))
    if args.device == "cuda":
        torch.cuda.set_device(local)
        if world > 1:
            dist.init_process_group("nccl", rank=rank, world_size=world, timeout=pg_timeout,
                                    device_id=torch.device("cuda", local))
    elif world > 1:
        dist.init_process_group("gloo", rank=rank, world_size=world, timeout=pg_timeout)
    return rank, world, local


def max_over_ranks(value: float, world: int, device: str = "cuda") -> float:
    import torch
    import torch.distributed as dist

    if world == 1:
        return value
    t = torch.tensor([value], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def barrier(world: int) -> None:
    import torch.distributed as dist

    if world > 1:
        dist.barrier()


def _sync(device: str) -> None:
    import torch

    if device == "cuda":
        torch.cuda.synchronize()


# ---------------------------------------------------------------------------
# The two arms
# ---------------------------------------------------------------------------


class Built:
    """What a benchmark loop needs from an arm: a step function and the layout around it."""

    def __init__(self, step, mesh, opt, graphable: bool, dp_rank: int, loss_holder: bool):
        self.step = step
        self.mesh = mesh
        self.opt = opt
        self.graphable = graphable
        self.dp_rank = dp_rank
        self.loss_holder = loss_holder  # this rank computes the loss (last pipeline stage)


def _import_arm(impl: str):
    """The ``minidist`` package of the requested arm (the reference one from baseline/_ref)."""
    if impl == "reference":
        sys.path.insert(0, REF_PATH)
        import minidist as md

        assert os.path.realpath(md.__file__).startswith(os.path.realpath(REF_PATH)), md.__file__
    else:
        import minidist as md

        assert os.path.realpath(md.__file__).startswith(os.path.realpath(os.path.join(ROOT, "minidist")))
    return md


def build(impl: str, c: dict, world: int, seed: int, graph: bool = False, device: str = "cuda",
          schedule: str = "1f1b") -> Built:
    """Model, optimizer and one training step through each framework's public API.

    Both arms follow the reference trainer's assembly (examples/train_gpt.py:120-218):
    a (tp, pp) mesh; GPT, or on a pipeline this stage's slice of
    ``build_pipeline_layers`` with a vocab-parallel cross-entropy on the last stage;
    DDP (25 MB buckets) or FSDP (one unit per Block, fp32 reduce) over the
    data-parallel group; AdamW.  Our arm differs only where its API offers the
    B200 path: FusedAdamW, deferred tail buckets, the fused LM-head loss and the
    in-kernel sharded AdamW of FSDP.
    """
    import torch
    from torch import nn

    md = _import_arm(impl)
    from minidist.models import GPT, Block, GPTConfig, build_pipeline_layers
    from minidist.tensor_parallel import vocab_parallel_cross_entropy

    ours = impl == "ours"
    dev = torch.device(device)
    cfg = GPTConfig(vocab_size=c["vocab"], block_size=c["seq"], n_layer=c["layers"], n_head=c["heads"],
                    n_embd=c["embd"], seed=seed)
    torch.manual_seed(seed)
    mesh = md.ParallelMesh(tp_size=c["tp"], pp_size=c["pp"])
    pipelined = c["pp"] > 1
    bf16 = device == "cuda"

    loss_fn = None
    if pipelined:
        layers = build_pipeline_layers(cfg, tp_group=mesh.tp_group, device=dev)
        mine = md.partition_layers(layers, mesh.pp_size, mesh.pp_rank)
        del layers
        vocab_start = mesh.tp_rank * (cfg.vocab_size // mesh.tp_size)
        if ours and mesh.is_last_stage:
            # The LM head's LayerNorm + GEMM + cross-entropy run as one fused loss.
            head = mine[-1]
            head.loss_only = True

            def loss_fn(hidden, targets):
                return head.loss(hidden, targets)

            core = nn.Sequential(*mine)
        else:
            def loss_fn(logits, targets):
                return vocab_parallel_cross_entropy(logits, targets, group=mesh.tp_group, vocab_start=vocab_start)

            core = nn.Sequential(*mine)
    else:
        core = GPT(cfg, tp_group=mesh.tp_group, device=dev)

    model = core
    if mesh.dp_size > 1 and c["strategy"] == "ddp":
        kw = dict(process_group=mesh.dp_group, bucket_cap_mb=25.0)
        if ours and not pipelined:
            # The tail buckets (the token-embedding gradient, produced last) finish their
            # all-reduce while FusedAdamW updates every other parameter.
            kw["defer_last_buckets"] = 2
        model = md.DistributedDataParallel(core, **kw)
    elif mesh.dp_size > 1 and c["strategy"] == "fsdp":
        kw = dict(unit_types=(Block,), process_group=mesh.dp_group,
                  mixed_precision=md.MixedPrecisionPolicy(param_dtype=torch.bfloat16 if bf16 else torch.float32,
                                                          reduce_dtype=torch.float32))
        model = md.FullyShardedDataParallel(core, **kw)

    if ours and device == "cuda":
        from minidist.optim import FusedAdamW

        opt = FusedAdamW(model.parameters(), lr=3e-4, capturable=graph)
    else:
        opt = torch.optim.AdamW(model.parameters(), lr=3e-4)

    if pipelined:
        stage = md.PipelineStage(model, mesh, loss_fn=loss_fn if mesh.is_last_stage else None)
        sched = md.build_schedule(schedule, stage, mesh, c["microbatches"])

        def step(ids, tgt):
            opt.zero_grad(set_to_none=True)
            ctx = model.no_sync() if hasattr(model, "no_sync") else _Null()
            with ctx, torch.autocast(device, dtype=torch.bfloat16, enabled=bf16):
                loss = sched.step(inputs=ids, targets=tgt)
            if hasattr(model, "finish_gradient_sync"):
                model.finish_gradient_sync()
            opt.step()
            return loss
    else:
        def step(ids, tgt):
            opt.zero_grad(set_to_none=True)
            # (No autocast weight-cast cache: a cached cast made during a graph capture
            # would outlive the capture.)
            with torch.autocast(device, dtype=torch.bfloat16, enabled=bf16, cache_enabled=not graph):
                _, loss = model(ids, tgt)
            loss.backward()
            opt.step()
            return loss

    graphable = ours and device == "cuda" and not pipelined and c["strategy"] != "fsdp"
    return Built(step, mesh, opt, graphable, mesh.dp_rank, mesh.is_last_stage)


class _Null:
    def __enter__(self):
        return None

    def __exit__(self, *exc):
        return False


def make_batches(n: int, c: dict, dp_rank: int, seed: int, pinned: bool, device: str = "cuda"):
    """Token batches seeded by ``seed + step*10000 + dp_rank`` (identical across TP/PP peers)."""
    import torch

    out = []
    for s in range(n):
        g = torch.Generator().manual_seed(seed + s * 10_000 + dp_rank)
        ids = torch.randint(0, c["vocab"], (c["batch"], c["seq"]), generator=g)
        tgt = torch.randint(0, c["vocab"], (c["batch"], c["seq"]), generator=g)
        if pinned and device == "cuda":
            out.append((ids.pin_memory(), tgt.pin_memory()))
        else:
            out.append((ids.to(device), tgt.to(device)))
    return out


def count_our_kernels(step, batch) -> int:
    """Kernels of this repository's native library launched by one step (namespace md::)."""
    import torch
    from torch.profiler import ProfilerActivity, profile

    with profile(activities=[ProfilerActivity.CUDA]) as prof:
        step(*batch)
        torch.cuda.synchronize()
    return sum(1 for e in prof.events() if e.device_type == torch.autograd.DeviceType.CUDA
               and "md::" in e.name)


def _loss_value(loss, built: Built, device: str) -> float:
    """The step's loss on every rank (pipeline: broadcast from the last stage, as the reference trainer does)."""
    import torch
    import torch.distributed as dist

    mesh = built.mesh
    if mesh.pp_size == 1:
        return float(loss.detach().float().item())
    v = torch.zeros(1, device=device)
    if loss is not None:
        v[0] = loss.detach().float().sum()
    dist.broadcast(v, src=mesh.pp_ranks[-1], group=mesh.pp_group)
    return float(v.item())


def main(argv=None) -> int:
    args = parse_args(argv)
    import torch

    if args.impl == "reference" and not os.path.isdir(os.path.join(REF_PATH, "minidist")):
        print(json.dumps({"impl": "reference", "unavailable": "baseline/_ref is not installed"}))
        return 0
    world_env = int(os.environ.get("WORLD_SIZE", "1"))
    c = resolve_config(args.config, world_env, args.tiny)
    if args.impl == "reference" and args.device == "cuda" and c["pp"] > 1 and args.schedule == "1f1b":
        # The reference's 1F1B (minidist/pipeline.py:205-231, 413-440 there) posts its
        # activation isend and its blocking gradient recv on the same NCCL process group, so
        # NCCL runs them in issue order on one stream: stage 0's send of microbatch m+1 waits
        # for stage 1's recv, which is queued behind stage 1's gradient send, which waits for
        # stage 0's recv, queued behind that first send.  Messages larger than NCCL's P2P
        # buffer (a 4 x 2048 x 2560 microbatch is 42 MB) therefore deadlock; on a B200 box the
        # 4-GPU run of this configuration made no progress for 4.5 minutes.  GPipe (all sends
        # of a direction before any recv of the other) has no such cycle.
        if int(os.environ.get("RANK", "0")) == 0:
            print(json.dumps({"impl": "reference", "unavailable": (
                "the reference's 1F1B schedule deadlocks on NCCL for this configuration (unbatched "
                "isend + blocking recv on one process group; 42 MB microbatch messages); "
                "--schedule gpipe runs the reference")}))
        return 0
    rank, world, local = setup(args)
    dev = args.device
    cuda = dev == "cuda"
    graph = args.impl == "ours" and not args.no_graph and cuda
    built = build(args.impl, c, world, args.seed, graph, dev, args.schedule)
    graph = graph and built.graphable
    step = built.step
    K, W = args.steps, args.warmup
    dev_batches = make_batches(K + W, c, built.dp_rank, args.seed, pinned=False, device=dev)
    graphed = None
    raw_step = step
    if graph:
        import minidist as md

        # Two eager steps (lazy initialisation), then one capture; the W warm-up
        # steps below are replays.  Every rank takes the graph or none does.
        ok = 1
        try:
            graphed = md.GraphedStep(step, dev_batches[0], warmup=2, optimizers=[built.opt])
        except Exception as exc:  # noqa: BLE001 -- report and run eagerly
            print(f"bench: CUDA-graph capture failed on rank {rank} ({exc!r}); running eagerly",
                  file=sys.stderr, flush=True)
            ok = 0
        if world > 1:
            import torch.distributed as dist

            flag = torch.tensor([ok], dtype=torch.int32, device="cuda")
            dist.all_reduce(flag, op=dist.ReduceOp.MIN)
            ok = int(flag.item())
        if ok:
            step = graphed
        else:
            if graphed is not None:
                graphed.release()
            graphed, graph = None, False

    # Clock sampling: one nvidia-smi per node (local rank 0) over every GPU of
    # this node's ranks, started before the warm-up so its start-up is over
    # when the timed window opens.
    sampler = None
    if cuda:
        uuid = "GPU-" + str(torch.cuda.get_device_properties(local).uuid)
        uuids = [uuid]
        if world > 1:
            import torch.distributed as dist

            allu = [None] * world
            dist.all_gather_object(allu, (os.uname().nodename, uuid))
            uuids = [u for n, u in allu if n == os.uname().nodename]
        sampler = ClockSampler(uuids) if local == 0 else None
        if sampler is not None:
            sampler.start()

    for i in range(W):
        step(*dev_batches[i])
    _sync(dev)
    barrier(world)
    _sync(dev)
    if cuda:
        t_start, t_end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        t_start.record()
    host_t0 = time.time()
    loss = None
    for i in range(K):
        loss = step(*dev_batches[W + i])
    if cuda:
        t_end.record()
    _sync(dev)
    host_t1 = time.time()
    barrier(world)
    clocks = sampler.stop(host_t0, host_t1) if sampler is not None else {"sm_mhz": None, "reasons": ["unsampled"]}
    if world > 1:
        import torch.distributed as dist

        got = [None] * world
        dist.all_gather_object(got, clocks)
        clocks = got[0]
    local_ms = t_start.elapsed_time(t_end) / K if cuda else (host_t1 - host_t0) * 1e3 / K
    ms = max_over_ranks(local_ms, world, dev)
    final_loss = _loss_value(loss, built, dev)

    tokens_per_step = c["batch"] * c["seq"] * built.mesh.dp_size
    e2e = None
    if not args.no_e2e:
        host_batches = make_batches(K, c, built.dp_rank, args.seed + 7, pinned=True, device=dev)
        barrier(world)
        _sync(dev)
        t0 = time.perf_counter()
        for ids_h, tgt_h in host_batches:
            ids = ids_h.to(dev, non_blocking=True)
            tgt = tgt_h.to(dev, non_blocking=True)
            _loss_value(step(ids, tgt), built, dev)  # device->host read of the step's loss
        _sync(dev)
        e2e_s = max_over_ranks(time.perf_counter() - t0, world, dev)
        e2e = {
            "value": tokens_per_step * K / e2e_s,
            "unit": "tokens/s",
            "h2d_bytes_per_step": int(host_batches[0][0].numel() * 8 * 2),
            "d2h_bytes_per_step": 4,
        }

    launches = 0
    if args.impl == "ours" and cuda:
        per_step = count_our_kernels(step, dev_batches[0])
        if per_step == 0 and graphed is not None:  # the profiler did not see inside the graph
            per_step = count_our_kernels(raw_step, dev_batches[0])
        launches = per_step * K
    if graphed is not None:
        graphed.release()

    value = tokens_per_step / (ms / 1e3)
    n, L, S, V = c["embd"], c["layers"], c["seq"], c["vocab"]
    # Training FLOPs per token: 6 x matmul parameters + causal attention (QK^T and PV, half the pairs).
    flops_tok = 6.0 * (L * 12 * n * n + n * V) + 6.0 * L * 2 * S * n
    par = f"dp{c['dp']}" if c["tp"] == 1 and c["pp"] == 1 else f"tp{c['tp']}xpp{c['pp']}xdp{c['dp']}"
    strategy = {"ddp": "ddp, 25 MB buckets overlapped with backward",
                "fsdp": "fsdp (ZeRO-3), bf16 parameter all-gather, fp32 master + fp32 reduce-scatter",
                "none": "no data parallelism"}[c["strategy"]]
    if c["strategy"] in ("ddp", "fsdp") and c["dp"] == 1:
        strategy += " (single replica: unwrapped)"
    cfg_out = {
        "name": args.config,
        "model": c["model"],
        "global_batch": c["batch"] * c["dp"],
        "seq_len": S,
        "parallelism": par,
        "strategy": strategy,
        "optimizer": "AdamW lr 3e-4",
        "cuda_graph": graph,
        "l2": "no flush: per-step working set (GBs of activations + weights) >> 126 MB L2",
    }
    if c["pp"] > 1:
        cfg_out["schedule"] = f"{args.schedule}, {c['microbatches']} microbatches"
    out = {
        "metric": METRIC,
        "value": value,
        "unit": "tokens/s",
        "n_gpus": world,
        "steps": K,
        "warmup": W,
        "ms_per_step": ms,
        "higher_is_better": True,
        "scaling": c["scaling"],
        "vs_baseline": None,
        "dtype": "bf16" if cuda else "fp32",
        "data": "synthetic uniform-random tokens (seeded), random-init weights",
        "config": cfg_out,
        "clocks": clocks,
        "e2e": e2e,
        "gpu_launches": launches,
        "tflops_per_gpu": flops_tok * tokens_per_step / world / (ms / 1e3) / 1e12,
        "final_loss": final_loss,
    }
    if args.tiny or not cuda:
        out["note"] = "wiring check: tiny model and/or CPU; not a benchmark number"
    if args.impl == "reference":
        out["impl"] = "reference"
    if rank == 0:
        print(json.dumps(out), flush=True)
    if world > 1:
        import torch.distributed as dist

        if args.impl == "ours" and cuda:
            from minidist.parallel import symm

            symm.release_all()
        dist.barrier()
        dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())
