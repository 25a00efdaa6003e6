"""Checkpoints in the reference's parameter format, sharded by (pipeline, tensor) rank.

The reference has no distributed checkpointing (README.md:413-414); its de
facto format is the unwrapped ``GPT.state_dict()`` (names such as
``blocks.3.attn.qkv.weight``, QKV rows interleaved per head) and, for
``FSDP``, the full parameters obtained through ``summon_full_params``
(fsdp.py:442-460).  This module writes exactly that format:

* ``save(dir, model, ...)`` — every (pp, tp) coordinate's data-parallel rank 0
  writes ``model_pp{p}_tp{t}.pt`` with its stage's full-precision parameters
  under unwrapped names (FSDP shards are gathered in fp32 first, so nothing is
  rounded to the gather dtype), each rank writes its optimizer state
  ``optim_rank{r}.pt``, and rank 0 writes ``manifest.json`` (mesh shape, step,
  scaler state, which file holds which names, how each tensor-parallel tensor
  is split).
* ``load(dir, model, ...)`` — the inverse, for the same mesh shape.
* ``consolidate(dir)`` — merges the shards on CPU into one unwrapped
  ``GPT.state_dict()`` (tensor-parallel shards concatenated, pipeline stages
  renumbered), loadable by the reference's ``GPT.load_state_dict`` and by ours.
"""

from __future__ import annotations

import json
import re
from pathlib import Path

import torch
import torch.distributed as dist
from torch import nn

from .. import comm

__all__ = ["save", "load", "consolidate", "full_state_dict"]

# How tensor parallelism splits each parameter (reference tensor_parallel.py:232-243, 297-301, 361-364, 402-407).
_TP_SPLIT = [
    (re.compile(r"attn\.qkv\.(weight|bias)$"), 0),
    (re.compile(r"mlp\.fc\.(weight|bias)$"), 0),
    (re.compile(r"head\.weight$"), 0),
    (re.compile(r"wte\.weight$"), 0),
    (re.compile(r"attn\.proj\.weight$"), 1),
    (re.compile(r"mlp\.proj\.weight$"), 1),
]


def _tp_dim(name: str) -> int | None:
    for pat, dim in _TP_SPLIT:
        if pat.search(name):
            return dim
    return None


def _unwrap(model: nn.Module) -> nn.Module:
    from ..ddp import DistributedDataParallel
    from ..fsdp import FullyShardedDataParallel
    from ..pipeline import PipelineStage

    while isinstance(model, (DistributedDataParallel, FullyShardedDataParallel, PipelineStage)):
        model = model.module
    return model


def full_state_dict(model: nn.Module) -> dict[str, torch.Tensor]:
    """This rank's (pp, tp) slice of the parameters in fp32 under unwrapped names (collective under FSDP)."""
    from ..fsdp import FullyShardedDataParallel

    if isinstance(model, FullyShardedDataParallel):
        names = {id(p): n for n, p in model.module.named_parameters()}
        out: dict[str, torch.Tensor] = {}
        for u in model._units:
            shard = u.flat_shard.detach().float()
            full = torch.empty(u.padded_numel, dtype=torch.float32, device=shard.device)
            comm.all_gather_into_tensor(full, shard.contiguous(), group=u.group)
            off = 0
            for p, n, shape in zip(u.params, u.numels, u.shapes):
                out[names[id(p)]] = full[off : off + n].view(shape).cpu().clone()
                off += n
        for n, b in model.module.named_buffers():
            out[n] = b.detach().cpu().clone()
        return out
    core = _unwrap(model)
    return {k: v.detach().float().cpu().clone() if v.is_floating_point() else v.detach().cpu().clone()
            for k, v in core.state_dict().items()}


def _mesh_coords(mesh):
    if mesh is None:
        return 0, 1, 0, 1, 0
    return mesh.pp_rank, mesh.pp_size, mesh.tp_rank, mesh.tp_size, mesh.dp_rank


def save(directory, model, optimizer=None, scaler=None, mesh=None, step: int = 0) -> Path:
    d = Path(directory)
    d.mkdir(parents=True, exist_ok=True)
    pp, npp, tp, ntp, dp = _mesh_coords(mesh)
    state = full_state_dict(model)  # collective for FSDP: every rank participates
    if dp == 0:
        torch.save(state, d / f"model_pp{pp}_tp{tp}.pt")
    if optimizer is not None:
        torch.save(optimizer.state_dict(), d / f"optim_rank{comm.get_rank()}.pt")
    names = sorted(state)
    gathered = [None] * comm.get_world_size()
    if comm.is_distributed() and comm.get_world_size() > 1:
        dist.all_gather_object(gathered, (pp, tp, dp, names))
    else:
        gathered = [(pp, tp, dp, names)]
    if comm.get_rank() == 0:
        files = {f"model_pp{p}_tp{t}.pt": n for (p, t, r, n) in gathered if r == 0}
        manifest = {
            "format": "minidist-gpt-v1",
            "step": step,
            "mesh": {"pp": npp, "tp": ntp, "world": comm.get_world_size()},
            "files": files,
            "tp_split": {k: _tp_dim(k) for fl in files.values() for k in fl},
            "scaler": scaler.state_dict() if scaler is not None else None,
        }
        (d / "manifest.json").write_text(json.dumps(manifest, indent=1))
    comm.barrier()
    return d


def load(directory, model, optimizer=None, scaler=None, mesh=None) -> dict:
    """Load a checkpoint written by :func:`save` with the same mesh shape; returns the manifest."""
    from ..fsdp import FullyShardedDataParallel

    d = Path(directory)
    manifest = json.loads((d / "manifest.json").read_text())
    pp, npp, tp, ntp, _ = _mesh_coords(mesh)
    if manifest["mesh"]["pp"] != npp or manifest["mesh"]["tp"] != ntp:
        raise ValueError(f"checkpoint mesh {manifest['mesh']} != current (pp={npp}, tp={ntp}); use consolidate()")
    state = torch.load(d / f"model_pp{pp}_tp{tp}.pt", map_location="cpu")
    if isinstance(model, FullyShardedDataParallel):
        names = {id(p): n for n, p in model.module.named_parameters()}
        with torch.no_grad():
            for u in model._units:
                flat = torch.cat([state[names[id(p)]].reshape(-1).float() for p in u.params])
                flat = torch.cat([flat, flat.new_zeros(u.padded_numel - u.total_numel)])
                lo = u.rank * u.shard_numel
                u.flat_shard.copy_(flat[lo : lo + u.shard_numel].to(u.flat_shard))
    else:
        core = _unwrap(model)
        own = core.state_dict()
        core.load_state_dict({k: v.to(own[k].dtype) for k, v in state.items()})
    if optimizer is not None:
        f = d / f"optim_rank{comm.get_rank()}.pt"
        if f.exists():
            optimizer.load_state_dict(torch.load(f, map_location="cpu"))
    if scaler is not None and manifest.get("scaler"):
        scaler.load_state_dict(manifest["scaler"])
    return manifest


def consolidate(directory) -> dict[str, torch.Tensor]:
    """Merge a sharded checkpoint into one unwrapped GPT state dict (CPU)."""
    d = Path(directory)
    manifest = json.loads((d / "manifest.json").read_text())
    npp, ntp = manifest["mesh"]["pp"], manifest["mesh"]["tp"]
    stages = []
    for p in range(npp):
        shards = [torch.load(d / f"model_pp{p}_tp{t}.pt", map_location="cpu") for t in range(ntp)]
        merged = {}
        for k in shards[0]:
            dim = _tp_dim(k)
            merged[k] = shards[0][k] if (dim is None or ntp == 1) else torch.cat([s[k] for s in shards], dim=dim)
        stages.append(merged)
    if npp == 1:
        return stages[0]
    # Pipeline stages hold nn.Sequential slices of [Embedding, Block x L, LMHead]
    # under keys "<index>.<rest>"; map them back to GPT names.
    out: dict[str, torch.Tensor] = {}
    layer = 0
    for st in stages:
        idx = sorted({int(k.split(".", 1)[0]) for k in st})
        for i in idx:
            sub = {k.split(".", 1)[1]: v for k, v in st.items() if k.split(".", 1)[0] == str(i)}
            if any(k.startswith("head.ln_f.") for k in sub):  # LM head wrapped for the fused loss
                sub = {k.removeprefix("head."): v for k, v in sub.items()}
            if any(k.startswith("wte.") or k == "wpe" for k in sub):
                out.update({f"embedding.{k}": v for k, v in sub.items()})
            elif any(k.startswith("ln_f.") for k in sub):
                out.update({f"lm_head.{k}": v for k, v in sub.items()})
            else:
                out.update({f"blocks.{layer}.{k}": v for k, v in sub.items()})
                layer += 1
    return out
