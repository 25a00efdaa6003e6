#!/usr/bin/env python3
"""Headline benchmark: GPT-2 small DDP training throughput (tokens/s for the whole job).

Config (the reference's DDP config): 12 layers, d_model 768, 12 heads, MLP
3072, vocab 50257, seq 1024, micro-batch 16 sequences per GPU, bf16 compute,
AdamW (lr 3e-4), 25 MB gradient buckets overlapped with backward, synthetic
uniform-random tokens from a seed, random-init weights.  Weak scaling: every
GPU runs the same per-GPU batch, data parallel over N GPUs.

    python bench.py                               # 1 GPU, our framework
    python bench.py --impl reference              # the unmodified reference (baseline/_ref)
    torchrun --nproc-per-node 8 bench.py --gpus 8 # one rank per GPU

Timing: W warm-up steps, then exactly K steps bracketed by a barrier and
torch.cuda.synchronize() on both sides, timed with CUDA events on the compute
stream; the reported step time is the maximum over ranks.  Every step's
working set (about 6 GB of activations plus 0.6 GB of fp32 weights) is far
larger than the 126 MB L2, so no explicit flush is needed.  SM clocks and
throttle reasons are sampled with nvidia-smi during the timed region.

Our arm runs the step as one CUDA graph (minidist.GraphedStep: forward,
backward, gradient all-reduce and FusedAdamW(capturable=True) captured once,
replayed per step, the step's token batch copied into the graph's input
buffers first); ``--no-graph`` runs the same step eagerly.

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

MODEL = dict(vocab=50257, layers=12, heads=12, embd=768, seq=1024, batch=16)
METRIC = "GPT train tokens/s/box at 1/2/4/8 B200 (DDP,FSDP,TP×PP×DP), max over ranks"


def parse_args():
    p = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=30)
    p.add_argument("--warmup", type=int, default=3)
    p.add_argument("--impl", choices=["ours", "reference"], default="ours")
    p.add_argument("--seed", type=int, default=1234)
    p.add_argument("--no-e2e", action="store_true")
    p.add_argument("--no-graph", action="store_true", help="our arm: run the step eagerly (no CUDA graph)")
    return p.parse_args()


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
    torch.cuda.set_device(local)
    if world > 1:
        os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
        dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=600),
                                device_id=torch.device("cuda", local))
    return rank, world, local


def max_over_ranks(value: float, world: int) -> float:
    import torch
    import torch.distributed as dist

    if world == 1:
        return value
    t = torch.tensor([value], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def barrier(world: int) -> None:
    import torch.distributed as dist

    if world > 1:
        dist.barrier()


# ---------------------------------------------------------------------------
# The two arms
# ---------------------------------------------------------------------------


def build(impl: str, world: int, seed: int, graph: bool = False):
    """Model, optimizer and a step function through each framework's public API."""
    import torch

    if impl == "reference":
        # The unmodified reference package, installed under baseline/_ref, on
        # its stock path: its GPT, its DDP, torch AdamW, bf16 autocast
        # (its examples/train_gpt.py with --precision bf16).
        sys.path.insert(0, REF_PATH)
        import minidist as md
        from minidist.models import GPT, GPTConfig

        assert os.path.realpath(md.__file__).startswith(os.path.realpath(REF_PATH)), md.__file__
        make_opt = lambda params: torch.optim.AdamW(params, lr=3e-4)  # noqa: E731
    else:
        import minidist as md
        from minidist.models import GPT, GPTConfig
        from minidist.optim import FusedAdamW

        assert os.path.realpath(md.__file__).startswith(os.path.realpath(os.path.join(ROOT, "minidist")))
        make_opt = lambda params: FusedAdamW(params, lr=3e-4, capturable=graph)  # noqa: E731

    cfg = GPTConfig(vocab_size=MODEL["vocab"], block_size=MODEL["seq"], n_layer=MODEL["layers"],
                    n_head=MODEL["heads"], n_embd=MODEL["embd"], seed=seed)
    torch.manual_seed(seed)
    # Pure data parallelism, as the reference trainer builds it: a (tp=1, pp=1)
    # mesh whose size-1 TP group keeps the whole model on every rank.
    mesh = md.ParallelMesh(tp_size=1, pp_size=1)
    model = GPT(cfg, tp_group=mesh.tp_group, device=torch.device("cuda"))
    if world > 1:
        # The last bucket (the token-embedding gradient, produced last in backward)
        # finishes its all-reduce while FusedAdamW updates every other parameter.
        model = md.DistributedDataParallel(model, process_group=mesh.dp_group, bucket_cap_mb=25.0,
                                           defer_last_buckets=2)
    opt = make_opt(model.parameters())

    def step(ids, tgt):
        opt.zero_grad(set_to_none=True)
        # (No autocast weight-cast cache: a cached cast made during a graph capture
        # would outlive the capture.)
        with torch.autocast("cuda", dtype=torch.bfloat16, cache_enabled=not graph):
            _, loss = model(ids, tgt)
        loss.backward()
        opt.step()
        return loss

    return cfg, model, opt, step


def make_batches(n: int, rank: int, seed: int, vocab: int, pinned: bool):
    import torch

    out = []
    for s in range(n):
        g = torch.Generator().manual_seed(seed + s * 10_000 + rank)
        ids = torch.randint(0, vocab, (MODEL["batch"], MODEL["seq"]), generator=g)
        tgt = torch.randint(0, vocab, (MODEL["batch"], MODEL["seq"]), generator=g)
        if pinned:
            out.append((ids.pin_memory(), tgt.pin_memory()))
        else:
            out.append((ids.cuda(), tgt.cuda()))
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


def main() -> int:
    args = parse_args()
    import torch

    if args.impl == "reference" and not os.path.isdir(os.path.join(REF_PATH, "minidist")):
        print(json.dumps({"impl": "reference", "unavailable": "baseline/_ref is not installed"}))
        return 0
    rank, world, local = setup(args)
    graph = args.impl == "ours" and not args.no_graph
    cfg, model, opt, step = build(args.impl, world, args.seed, graph)
    K, W = args.steps, args.warmup
    dev_batches = make_batches(K + W, rank, args.seed, cfg.vocab_size, pinned=False)
    graphed = None
    raw_step = step
    if graph:
        import minidist as md

        # Two eager steps (lazy initialisation), then one capture; the W warm-up
        # steps below are replays.  Every rank takes the graph or none does.
        ok = 1
        try:
            graphed = md.GraphedStep(step, dev_batches[0], warmup=2, optimizers=[opt])
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
    torch.cuda.synchronize()
    barrier(world)
    torch.cuda.synchronize()
    t_start, t_end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    host_t0 = time.time()
    t_start.record()
    loss = None
    for i in range(K):
        loss = step(*dev_batches[W + i])
    t_end.record()
    torch.cuda.synchronize()
    host_t1 = time.time()
    barrier(world)
    clocks = sampler.stop(host_t0, host_t1) if sampler is not None else None
    if world > 1:
        import torch.distributed as dist

        got = [None] * world
        dist.all_gather_object(got, clocks)
        clocks = got[0]
    ms = max_over_ranks(t_start.elapsed_time(t_end) / K, world)
    final_loss = float(loss.detach().float().item())

    e2e = None
    if not args.no_e2e:
        host_batches = make_batches(K, rank, args.seed + 7, cfg.vocab_size, pinned=True)
        barrier(world)
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        for ids_h, tgt_h in host_batches:
            ids = ids_h.to("cuda", non_blocking=True)
            tgt = tgt_h.to("cuda", non_blocking=True)
            _ = step(ids, tgt).item()  # device->host read of the step's loss
        torch.cuda.synchronize()
        e2e_s = max_over_ranks(time.perf_counter() - t0, world)
        tokens = MODEL["batch"] * MODEL["seq"] * world * K
        e2e = {
            "value": tokens / e2e_s,
            "unit": "tokens/s",
            "h2d_bytes_per_step": int(host_batches[0][0].numel() * 8 * 2),
            "d2h_bytes_per_step": 4,
        }

    launches = 0
    if args.impl == "ours":
        per_step = count_our_kernels(step, dev_batches[0])
        if per_step == 0 and graphed is not None:  # the profiler did not see inside the graph
            per_step = count_our_kernels(raw_step, dev_batches[0])
        launches = per_step * K
    if graphed is not None:
        graphed.release()

    tokens_per_step = MODEL["batch"] * MODEL["seq"] * world
    value = tokens_per_step / (ms / 1e3)
    # Training FLOPs per token: 6 x matmul parameters + causal attention (QK^T and PV, half the pairs).
    n, L, S = MODEL["embd"], MODEL["layers"], MODEL["seq"]
    flops_tok = 6.0 * (L * 12 * n * n + n * MODEL["vocab"]) + 6.0 * L * 2 * S * n
    out = {
        "metric": METRIC,
        "value": value,
        "unit": "tokens/s",
        "n_gpus": world,
        "steps": K,
        "warmup": W,
        "ms_per_step": ms,
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "bf16",
        "data": "synthetic uniform-random tokens (seeded), random-init weights",
        "config": {
            "model": "gpt2-small 12L/768d/12h, vocab 50257 (untied head)",
            "global_batch": MODEL["batch"] * world,
            "seq_len": MODEL["seq"],
            "parallelism": f"dp{world}",
            "strategy": "ddp, 25 MB buckets overlapped with backward",
            "optimizer": "AdamW lr 3e-4",
            "cuda_graph": graph,
            "l2": "no flush: per-step working set (~6 GB activations + weights) >> 126 MB L2",
        },
        "clocks": clocks,
        "e2e": e2e,
        "gpu_launches": launches,
        "tflops_per_gpu": flops_tok * tokens_per_step / world / (ms / 1e3) / 1e12,
        "final_loss": final_loss,
    }
    if args.impl == "reference":
        out["impl"] = "reference"
    if rank == 0:
        print(json.dumps(out), flush=True)
    if world > 1:
        import torch.distributed as dist

        if args.impl == "ours":
            from minidist.parallel import symm

            symm.release_all()
        dist.barrier()
        dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())
