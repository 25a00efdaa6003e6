"""minidist for B200 — 3-D parallel GPT training with hand-written sm_100a kernels.

Same public API as the reference ``minidist`` package (reference
minidist/__init__.py:17-85): data parallelism (:mod:`minidist.ddp`), ZeRO-3
(:mod:`minidist.fsdp`), Megatron tensor parallelism
(:mod:`minidist.tensor_parallel`), GPipe/1F1B pipelines
(:mod:`minidist.pipeline`), mixed precision with a collective loss scaler
(:mod:`minidist.amp`) and profiling/overlap analysis
(:mod:`minidist.profiling`), composed on a :class:`~minidist.mesh.ParallelMesh`.

What is new underneath: the GPT hot path runs on hand-written sm_100a kernels
(:mod:`minidist.ops`: tcgen05/TMEM GEMMs with fused epilogues, flash attention,
LayerNorm, fused cross-entropy, multi-tensor AdamW) and the gradient and
tensor-parallel collectives run as peer-memory kernels over NVLink
(:mod:`minidist.parallel`), with NCCL kept for pipeline point-to-point traffic
and as the fallback.
"""

from .amp import DistributedGradScaler, PrecisionConfig, resolve_precision
from .comm import (
    barrier,
    comm_stats,
    get_rank,
    get_world_size,
    init_distributed,
    is_primary,
    print_rank0,
    record_comm,
    shutdown_distributed,
)
from .ddp import DDP, DistributedDataParallel
from .fsdp import FSDP, FullyShardedDataParallel, MixedPrecisionPolicy
from .graphs import GraphedStep
from .mesh import ParallelMesh
from .pipeline import PipelineStage, build_schedule, partition_layers, theoretical_bubble_fraction
from .profiling import analyze_trace, format_collective_table, profile_steps, summarize_collectives
from .tensor_parallel import (
    ColumnParallelLinear,
    RowParallelLinear,
    VocabParallelEmbedding,
    vocab_parallel_cross_entropy,
)

__version__ = "0.1.0"

__all__ = [
    "GraphedStep",
    "DDP",
    "DistributedDataParallel",
    "FSDP",
    "FullyShardedDataParallel",
    "MixedPrecisionPolicy",
    "ParallelMesh",
    "PipelineStage",
    "ColumnParallelLinear",
    "RowParallelLinear",
    "VocabParallelEmbedding",
    "DistributedGradScaler",
    "PrecisionConfig",
    "vocab_parallel_cross_entropy",
    "build_schedule",
    "partition_layers",
    "theoretical_bubble_fraction",
    "resolve_precision",
    "init_distributed",
    "shutdown_distributed",
    "barrier",
    "get_rank",
    "get_world_size",
    "is_primary",
    "print_rank0",
    "comm_stats",
    "record_comm",
    "profile_steps",
    "summarize_collectives",
    "format_collective_table",
    "analyze_trace",
    "__version__",
]
