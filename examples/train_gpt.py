#!/usr/bin/env python3
"""Train a GPT under any combination of tensor, pipeline and data parallelism.

Flags match the reference trainer (examples/train_gpt.py:59-92):

    torchrun --nproc-per-node 8 examples/train_gpt.py --strategy ddp --precision bf16
    torchrun --nproc-per-node 8 examples/train_gpt.py --strategy fsdp --fsdp-param-dtype bf16
    torchrun --nproc-per-node 8 examples/train_gpt.py --tp 2 --pp 2 --strategy ddp --microbatches 8
    torchrun --nproc-per-node 4 examples/train_gpt.py --tp 2 --backend gloo        # CPU wiring check

On B200 with ``--precision bf16`` every block runs on the hand-written sm_100a
kernels and gradients are averaged by the peer-memory all-reduce; with
``--precision fp32`` (or on CPU) the portable path runs.  Added flags:
``--optimizer {auto,fused,torch}`` and ``--timing {device,host}`` (device =
CUDA-event step time, maximum over ranks, the default on GPU).

The data are synthetic uniform-random tokens, seeded by
``seed + step*10000 + dp_rank`` so tensor/pipeline peers see identical batches
and data-parallel replicas different ones; the loss should hover near
``ln(vocab)``.
"""

from __future__ import annotations

import argparse
import json
import os
import sys
import time
from pathlib import Path

import torch
from torch import nn

sys.path.insert(0, str(Path(__file__).resolve().parent.parent))

from minidist import (  # noqa: E402
    DistributedDataParallel,
    DistributedGradScaler,
    FullyShardedDataParallel,
    ParallelMesh,
    PipelineStage,
    analyze_trace,
    barrier,
    build_schedule,
    format_collective_table,
    init_distributed,
    partition_layers,
    print_rank0,
    profile_steps,
    resolve_precision,
    shutdown_distributed,
    summarize_collectives,
)
from minidist.fsdp import MixedPrecisionPolicy  # noqa: E402
from minidist.models import GPT, Block, GPTConfig, LMHead, build_pipeline_layers  # noqa: E402
from minidist.tensor_parallel import vocab_parallel_cross_entropy  # noqa: E402


def parse_args(argv=None) -> argparse.Namespace:
    p = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    mesh = p.add_argument_group("mesh")
    mesh.add_argument("--tp", type=int, default=1, help="tensor-parallel degree")
    mesh.add_argument("--pp", type=int, default=1, help="pipeline-parallel degree")
    mesh.add_argument("--backend", default=None, choices=[None, "nccl", "gloo"])
    strat = p.add_argument_group("strategy")
    strat.add_argument("--strategy", default="ddp", choices=["none", "ddp", "fsdp"])
    strat.add_argument("--schedule", default="1f1b", choices=["gpipe", "1f1b"])
    strat.add_argument("--microbatches", type=int, default=4)
    strat.add_argument("--precision", default="fp32", choices=["fp32", "fp16", "bf16", "auto"])
    strat.add_argument("--fsdp-param-dtype", default=None, choices=[None, "bf16", "fp16"])
    strat.add_argument("--bucket-cap-mb", type=float, default=25.0)
    strat.add_argument("--no-overlap", action="store_true", help="disable DDP backward/all-reduce overlap")
    model = p.add_argument_group("model")
    model.add_argument("--layers", type=int, default=8)
    model.add_argument("--heads", type=int, default=8)
    model.add_argument("--embd", type=int, default=512)
    model.add_argument("--vocab", type=int, default=8192)
    model.add_argument("--seq-len", type=int, default=256)
    model.add_argument("--batch-size", type=int, default=16, help="per data-parallel replica")
    run = p.add_argument_group("run")
    run.add_argument("--steps", type=int, default=20)
    run.add_argument("--lr", type=float, default=3e-4)
    run.add_argument("--seed", type=int, default=1234)
    run.add_argument("--profile", metavar="PATH", default=None,
                     help="export a Chrome trace (one per rank) and print an overlap report")
    run.add_argument("--optimizer", default="auto", choices=["auto", "fused", "torch"],
                     help="AdamW implementation (fused = multi-tensor sm_100a kernel)")
    run.add_argument("--timing", default="auto", choices=["auto", "device", "host"])
    run.add_argument("--save", metavar="DIR", default=None, help="write a checkpoint here at the end")
    run.add_argument("--kernels", default="fused", choices=["fused", "nccl"],
                     help="fused: peer-memory collectives fused into the kernels; nccl: the same model with "
                          "every collective through NCCL (A/B comparison)")
    run.add_argument("--metrics-jsonl", metavar="PATH", default=None,
                     help="append one JSON line per logged step and a summary line (rank 0)")
    run.add_argument("--defer-last-buckets", type=int, default=0, metavar="K",
                     help="DDP: let the all-reduce of the last K gradient buckets (the token embedding, "
                          "produced last) finish under the optimizer step instead of inside backward")
    run.add_argument("--cuda-graph", action="store_true",
                     help="capture the whole training step (forward, backward, collectives, FusedAdamW) as "
                          "one CUDA graph and replay it (no pipeline, no FSDP, bf16 without loss scaling)")
    return p.parse_args(argv)


class _MetricsSink:
    """JSON-lines metrics (rank 0 only): per logged step, then one summary record."""

    def __init__(self, path: str | None, rank: int):
        self.f = open(path, "a") if (path and rank == 0) else None

    def write(self, **rec) -> None:
        if self.f is not None:
            self.f.write(json.dumps(rec) + "\n")
            self.f.flush()

    def close(self) -> None:
        if self.f is not None:
            self.f.close()


def make_batch(config: GPTConfig, batch_size: int, dp_rank: int, step: int, seed: int, device):
    g = torch.Generator().manual_seed(seed + step * 10_000 + dp_rank)
    ids = torch.randint(0, config.vocab_size, (batch_size, config.block_size), generator=g)
    targets = torch.randint(0, config.vocab_size, (batch_size, config.block_size), generator=g)
    if device.type == "cuda":
        ids, targets = ids.pin_memory(), targets.pin_memory()
    return ids.to(device, non_blocking=True), targets.to(device, non_blocking=True)


def build(args, mesh: ParallelMesh, config: GPTConfig, device, precision):
    loss_fn = None
    fused = device.type == "cuda" and precision.enabled and precision.dtype == torch.bfloat16
    if mesh.pp_size > 1:
        layers = build_pipeline_layers(config, tp_group=mesh.tp_group, device=device)
        mine = partition_layers(layers, mesh.pp_size, mesh.pp_rank)
        vocab_start = mesh.tp_rank * (config.vocab_size // mesh.tp_size)
        if fused and isinstance(mine[-1], LMHead):
            # LayerNorm + head GEMM + cross-entropy as one fused loss on the last stage.
            head = mine[-1]
            head.loss_only = True

            def loss_fn(hidden, targets):
                return head.loss(hidden, targets)
        else:
            def loss_fn(logits, targets):
                return vocab_parallel_cross_entropy(logits, targets, group=mesh.tp_group, vocab_start=vocab_start)
        core: nn.Module = nn.Sequential(*mine)
    else:
        core = GPT(config, tp_group=mesh.tp_group, device=device)

    wrapped = core
    if mesh.dp_size > 1 and args.strategy == "ddp":
        wrapped = DistributedDataParallel(core, process_group=mesh.dp_group, bucket_cap_mb=args.bucket_cap_mb,
                                          overlap_with_backward=not args.no_overlap,
                                          defer_last_buckets=args.defer_last_buckets)
    elif mesh.dp_size > 1 and args.strategy == "fsdp":
        param_dtype = {None: torch.float32, "bf16": torch.bfloat16, "fp16": torch.float16}[args.fsdp_param_dtype]
        wrapped = FullyShardedDataParallel(
            core, unit_types=(Block,), process_group=mesh.dp_group,
            mixed_precision=MixedPrecisionPolicy(param_dtype=param_dtype, reduce_dtype=torch.float32))
    return wrapped, core, loss_fn


def make_optimizer(args, model, device):
    params = list(model.parameters())
    use_fused = args.optimizer == "fused" or args.cuda_graph or (
        args.optimizer == "auto" and device.type == "cuda" and all(p.dtype == torch.float32 for p in params))
    if use_fused:
        from minidist.optim import FusedAdamW

        return FusedAdamW(params, lr=args.lr, capturable=args.cuda_graph)
    return torch.optim.AdamW(params, lr=args.lr)


def _broadcast_loss(loss, mesh: ParallelMesh, device) -> float:
    value = torch.zeros(1, device=device)
    if loss is not None:
        value[0] = loss.sum()
    if mesh.pp_size > 1:
        torch.distributed.broadcast(value, src=mesh.pp_ranks[-1], group=mesh.pp_group)
    return float(value.item())


def _max_over_ranks(x: float, device) -> float:
    if torch.distributed.is_initialized() and torch.distributed.get_world_size() > 1:
        t = torch.tensor([x], dtype=torch.float64, device=device)
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
        return float(t.item())
    return x


def main(argv=None) -> None:
    args = parse_args(argv)
    if args.kernels == "nccl":
        # Read when the communicators, reducers and fused paths are first set up.
        for var in ("MINIDIST_PEER_MEMORY", "MINIDIST_TP_FUSED", "MINIDIST_FSDP_FUSED"):
            os.environ[var] = "0"
    rank, world, device = init_distributed(backend=args.backend)
    metrics = _MetricsSink(args.metrics_jsonl, rank)
    torch.manual_seed(args.seed)
    mesh = ParallelMesh(tp_size=args.tp, pp_size=args.pp)
    config = GPTConfig(vocab_size=args.vocab, block_size=args.seq_len, n_layer=args.layers, n_head=args.heads,
                       n_embd=args.embd, seed=args.seed)
    precision = resolve_precision(args.precision, device)
    device_timing = args.timing == "device" or (args.timing == "auto" and device.type == "cuda")

    print_rank0(f"\n{'=' * 74}")
    print_rank0(f"  {mesh.describe()}")
    print_rank0(f"  model: {config.n_layer}L x {config.n_embd}d x {config.n_head}h, vocab {config.vocab_size}, "
                f"seq {config.block_size} ({config.param_count() / 1e6:.1f}M params)")
    print_rank0(f"  strategy: {args.strategy}  precision: {precision}  "
                + (f"pipeline: {args.schedule} x{args.microbatches}" if mesh.pp_size > 1 else ""))
    print_rank0("=" * 74)

    model, core, loss_fn = build(args, mesh, config, device, precision)
    optimizer = make_optimizer(args, model, device)
    scaler = DistributedGradScaler(enabled=precision.needs_grad_scaler)
    schedule = None
    if mesh.pp_size > 1:
        stage = PipelineStage(model, mesh, loss_fn=loss_fn if mesh.is_last_stage else None)
        schedule = build_schedule(args.schedule, stage, mesh, args.microbatches)
    if isinstance(model, FullyShardedDataParallel):
        s = model.memory_summary()
        print_rank0(f"  FSDP: {s['num_units']} units, {s['shard_params_MB']:.1f}MB/rank sharded vs "
                    f"{s['replicated_params_MB']:.1f}MB replicated; transient gather {s['transient_gather_MB']:.1f}MB")
    if isinstance(model, DistributedDataParallel):
        print_rank0(f"  DDP: {len(model.bucket_summary())} buckets, reducer={model.reducer_name}")

    graphed = None
    if args.cuda_graph:
        if schedule is not None or isinstance(model, FullyShardedDataParallel) or scaler.enabled \
                or device.type != "cuda":
            raise SystemExit("--cuda-graph needs CUDA, no pipeline, no FSDP and no fp16 loss scaling")
        from minidist import GraphedStep

        def graph_body(ids, targets):
            optimizer.zero_grad(set_to_none=True)
            # No autocast weight-cast cache: a cast cached during capture would outlive it.
            with torch.autocast("cuda", dtype=precision.dtype, enabled=precision.enabled, cache_enabled=False):
                _, loss = model(ids, targets)
            loss.backward()
            optimizer.step()
            return loss

        # Two eager steps on a side stream (lazy set-up), then one capture.
        graphed = GraphedStep(graph_body, make_batch(config, args.batch_size, mesh.dp_rank, 0, args.seed, device),
                              warmup=2, optimizers=[optimizer])

    def train_step(step: int) -> float:
        ids, targets = make_batch(config, args.batch_size, mesh.dp_rank, step, args.seed, device)
        if graphed is not None:
            return float(graphed(ids, targets).item())
        optimizer.zero_grad(set_to_none=True)
        if schedule is not None:
            schedule.loss_scale = scaler.scale
            sync_ctx = model.no_sync() if hasattr(model, "no_sync") else _null()
            with sync_ctx, precision.autocast():
                loss = schedule.step(inputs=ids, targets=targets)
            if hasattr(model, "finish_gradient_sync"):
                model.finish_gradient_sync()
            value = _broadcast_loss(loss, mesh, device)
        else:
            with precision.autocast():
                _, loss = model(ids, targets)
            scaler.scale_loss(loss).backward()
            value = float(loss.detach())
        scaler.step(optimizer)
        scaler.update()
        return value

    train_step(0)  # warm-up: communicator creation, allocator growth, kernel attributes
    if device.type == "cuda":
        torch.cuda.synchronize()
        torch.cuda.reset_peak_memory_stats()
    barrier()

    tokens_per_step = args.batch_size * config.block_size * mesh.dp_size
    ev0 = ev1 = None
    if device_timing:
        ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        ev0.record()
    start = time.perf_counter()
    for step in range(1, args.steps + 1):
        loss = train_step(step)
        if step % max(1, args.steps // 10) == 0:
            el = time.perf_counter() - start
            print_rank0(f"  step {step:>4}/{args.steps}  loss {loss:>7.4f}  {el / step * 1e3:>7.1f} ms/step  "
                        f"{tokens_per_step * step / el:>9.0f} tok/s")
            metrics.write(step=step, loss=loss, ms_per_step=el / step * 1e3, tokens_per_s=tokens_per_step * step / el,
                          timing="host, rank 0")
    if device.type == "cuda":
        torch.cuda.synchronize()
    total = time.perf_counter() - start
    if device_timing:
        ev1.record()
        ev1.synchronize()
        total = ev0.elapsed_time(ev1) / 1e3
    total = _max_over_ranks(total, device)
    kind = "device time, max over ranks" if device_timing else "host time, max over ranks"
    print_rank0(f"\n  {args.steps} steps in {total:.2f}s ({total / args.steps * 1e3:.1f} ms/step, "
                f"{tokens_per_step * args.steps / total:.0f} tok/s; {kind})")
    metrics.write(event="summary", steps=args.steps, ms_per_step=total / args.steps * 1e3,
                  tokens_per_s=tokens_per_step * args.steps / total, timing=kind, kernels=args.kernels,
                  peak_mem_gib=(torch.cuda.max_memory_allocated() / 1024**3 if device.type == "cuda" else None))
    metrics.close()
    if device.type == "cuda":
        print_rank0(f"  peak memory: {torch.cuda.max_memory_allocated() / 1024**3:.2f} GiB/rank")
    if scaler.enabled:
        print_rank0(f"  {scaler.summary()}")
    if schedule is not None:
        r = schedule.report()
        print_rank0(f"  pipeline bubble: measured {r['measured_bubble'] * 100:.1f}%  "
                    f"theoretical {r['theoretical_bubble'] * 100:.1f}%  (stage {mesh.pp_rank})")
    if args.save:
        from minidist.utils import checkpoint

        path = checkpoint.save(args.save, model, optimizer=optimizer, scaler=scaler, mesh=mesh, step=args.steps)
        print_rank0(f"  checkpoint -> {path}")
    if args.profile:
        trace = Path(args.profile)
        trace = trace.with_name(f"{trace.stem}_rank{mesh.rank}{trace.suffix or '.json'}")
        print_rank0(f"\n  profiling -> {trace.parent}/{trace.stem[:-6]}_rank*.json")
        prof = profile_steps(lambda s: train_step(s + 1000), num_steps=6, trace_path=trace)
        print_rank0("\n  collectives:")
        print_rank0(format_collective_table(summarize_collectives(prof)))
        barrier()
        if mesh.rank == 0:
            print_rank0("\n  overlap:")
            print_rank0(analyze_trace(trace).format())
    if graphed is not None:
        graphed.release()  # a graph holding peer-memory or NCCL work goes before the process group
    shutdown_distributed()


class _null:
    def __enter__(self):
        return None

    def __exit__(self, *exc):
        return False


if __name__ == "__main__":
    main()
