"""Fused B200 execution of the GPT modules.

Each transformer block, the embedding and the LM head run as one autograd
node whose forward and backward call the hand-written sm_100a kernels:

forward of a block (``M = batch*seq`` rows, bf16 activations)::

    h1, mu1, r1 = LayerNorm(x)                      md_ln_fwd
    qkv         = h1 Wqkv^T + bqkv                  tcgen05 GEMM, bias epilogue
    y, lse      = causal attention(qkv)             md_attn_fwd
    x1          = x + y Wproj^T + bproj             GEMM, bias + residual epilogue
    h2, mu2, r2 = LayerNorm(x1)
    a, hpre     = GELU(h2 Wfc^T + bfc)              GEMM, bias + GELU epilogue
    x2          = x1 + a Wmproj^T + bmproj          GEMM, bias + residual epilogue

backward: weight gradients come straight out of the wgrad GEMM epilogue in
fp32 (accumulating when a gradient already exists), GELU' is fused into the
data-gradient GEMM of the MLP projection, the two row-parallel bias gradients
are column sums fused into the LayerNorm backward, and nothing goes through
autograd's AccumulateGrad; wrappers learn that a gradient is ready through
:mod:`minidist.ops.grads`.

With tensor parallelism every reduction over the TP group (the reference's
``g`` and ``f``, tensor_parallel.py:134-172) runs in a peer-memory kernel of
:mod:`minidist.parallel.collectives` when the group shares a node:

* row-parallel forward (attention and MLP projections): ``md_gemm_ar``, the
  GEMM with its all-reduce, bias and residual in one persistent kernel;
* column-parallel backward (QKV, fc and the LM head's data gradient): the same
  kernel on the data-gradient GEMM;
* vocab-parallel embedding forward: ``md_embed_tp``, which reads each token
  row from the rank that owns it instead of reducing masked lookups;
* vocab-parallel cross-entropy statistics: ``md_ce_tp``.

NCCL (``collectives.all_reduce_``) is the fallback off-node.
"""

from __future__ import annotations

import os

import torch

from .. import comm
from ..ops import _native as nat
from ..ops import gemm as G
from ..ops import grads as gradsink
from ..ops import kernels as K

_SHADOW = "_md_bf16"
_SHADOW_VER = "_md_bf16_ver"


def enabled() -> bool:
    return os.environ.get("MINIDIST_FUSED", "1") not in ("0", "false", "no")


def should_fuse(x: torch.Tensor) -> bool:
    """Take the fused path for CUDA tensors under bf16 autocast, or for bf16 activations."""
    if not x.is_cuda or not enabled():
        return False
    if torch.is_autocast_enabled("cuda") and torch.get_autocast_dtype("cuda") == torch.bfloat16:
        return nat.available() or _missing_library()
    return x.dtype == torch.bfloat16 and (nat.available() or _missing_library())


def _missing_library() -> bool:
    # On a CUDA machine the kernels are not optional: fail loudly.
    raise nat.NativeError(f"minidist native library not found at {nat.library_path()}; run `python -m minidist._build`")


# ---------------------------------------------------------------------------
# Parameters: bf16 shadows for the GEMMs, fp32 gradient destinations
# ---------------------------------------------------------------------------


def bf16_weight(p: torch.Tensor) -> torch.Tensor:
    """bf16 view of parameter ``p`` (a cached shadow for fp32 masters, refreshed when ``p`` changes)."""
    if p.dtype == torch.bfloat16:
        return p.detach() if p.is_contiguous() else p.detach().contiguous()
    sh = getattr(p, _SHADOW, None)
    ver = p._version
    if sh is None or sh.shape != p.shape or getattr(p, _SHADOW_VER, None) != ver:
        if sh is None or sh.shape != p.shape:
            sh = torch.empty(p.shape, dtype=torch.bfloat16, device=p.device)
            setattr(p, _SHADOW, sh)
        sh.copy_(p.detach())
        setattr(p, _SHADOW_VER, ver)
    return sh


_SHADOW_LIST = "_md_shadow_params"


def refresh_shadows(module: torch.nn.Module) -> None:
    """Bring every stale bf16 weight shadow of ``module`` up to date in ONE multi-tensor launch
    (the AdamW kernel in shadow-only mode) instead of one cast per weight: on the first
    forward, and after any optimizer that does not refresh the shadows itself (FusedAdamW
    does, inside its update) has changed the fp32 weights."""
    params = getattr(module, _SHADOW_LIST, None)
    if params is None:
        params = [p for p in module.parameters() if p.dim() == 2 and p.dtype == torch.float32 and p.is_cuda
                  and p.is_contiguous()]
        setattr(module, _SHADOW_LIST, params)
    # (Parameters whose storage is released -- FSDP units between their gathers -- are skipped;
    # bf16_weight refreshes them when their unit runs.)
    stale = [p for p in params if (getattr(p, _SHADOW_VER, None) != p._version
                                   or getattr(p, _SHADOW, None) is None or getattr(p, _SHADOW).shape != p.shape)
             and p.untyped_storage().nbytes() >= (p.storage_offset() + p.numel()) * 4]
    if len(stale) < 2:
        return  # nothing to batch; bf16_weight handles a single one
    rows, chunks = [], []
    chunk = nat.lib().md_adamw_chunk()
    for i, p in enumerate(stale):
        sh = getattr(p, _SHADOW, None)
        if sh is None or sh.shape != p.shape:
            sh = torch.empty(p.shape, dtype=torch.bfloat16, device=p.device)
            setattr(p, _SHADOW, sh)
        ptr = p.data_ptr()
        rows.append((ptr, ptr, ptr, ptr, sh.data_ptr(), p.numel()))
        chunks += [(i, c) for c in range(-(-p.numel() // chunk))]
    dev = stale[0].device
    table = torch.tensor(rows, dtype=torch.int64).pin_memory().to(dev, non_blocking=True)
    chunk_t = torch.tensor(chunks, dtype=torch.int32).pin_memory().to(dev, non_blocking=True)
    rc = nat.lib().md_adamw(table.data_ptr(), chunk_t.data_ptr(), len(chunks), 0.0, 0.0, 0.0, 0.0, 0.0, 1.0, 1.0,
                            None, None, 1, nat.stream_ptr(), None)
    nat.check(rc, "md_adamw(shadows)")
    # (The pinned host tables are released through torch's caching host allocator, which keeps a
    # block until the copy that reads it has run.)
    for p in stale:
        setattr(p, _SHADOW_VER, p._version)


def fp32_param(p: torch.Tensor) -> torch.Tensor:
    """fp32, contiguous, 16-byte-aligned copy or view of a (small) parameter such as a bias or LN weight."""
    t = p.detach()
    if t.dtype != torch.float32:
        return t.float()  # a fresh (aligned, contiguous) fp32 tensor
    if not t.is_contiguous() or (t.data_ptr() % 16):
        t = t.contiguous().clone()
    return t


def _fp32_params(*params):
    """``fp32_param`` of several small parameters (None passes through).  Low-precision ones (FSDP
    views gathered in bf16) are converted together -- one concatenation and one cast -- and
    returned as views of the result (each slice starts 16-byte aligned)."""
    low = [p for p in params if p is not None and p.dtype != torch.float32]
    if len(low) < 2:
        return tuple(None if p is None else fp32_param(p) for p in params)
    pads = []
    for p in low:
        n = p.numel()
        pads.append(p.detach().reshape(-1))
        if n % 4:
            pads.append(p.new_zeros(4 - n % 4))
    flat = torch.cat(pads).float()
    out, off = [], 0
    views = {}
    for p in low:
        n = p.numel()
        views[id(p)] = flat[off: off + n].view(p.shape)
        off += -(-n // 4) * 4
    for p in params:
        if p is None:
            out.append(None)
        elif id(p) in views:
            out.append(views[id(p)])
        else:
            out.append(fp32_param(p))
    return tuple(out)


class _GradTarget:
    """Where a kernel writes ``p``'s fp32 gradient; :meth:`commit` publishes it."""

    __slots__ = ("p", "dst", "accumulate", "_tmp")

    def __init__(self, p: torch.Tensor):
        self.p = p
        self._tmp = None
        mg = gradsink.main_grad(p)
        if (p.dtype != torch.float32 and p.grad is None and mg is not None and mg.dtype == torch.float32
                and mg.is_contiguous() and mg.data_ptr() % 16 == 0):
            # A low-precision parameter (an FSDP view gathered in bf16) whose wrapper keeps an fp32
            # gradient buffer: the kernel writes there directly (no bf16 round trip); the first
            # write of a backward overwrites, later ones accumulate.
            self.dst, self.accumulate = mg, bool(getattr(p, "_md_grad_written", False))
            p._md_grad_written = True
            return
        if p.dtype == torch.float32 and (p.grad is None or p.grad.is_contiguous()):
            self.dst, self.accumulate = gradsink.grad_destination(p)
            if not self.dst.is_contiguous() or self.dst.data_ptr() % 16:
                self._tmp = torch.empty(p.shape, dtype=torch.float32, device=p.device)
                self.dst, self.accumulate = self._tmp, False
        else:
            self._tmp = torch.empty(p.shape, dtype=torch.float32, device=p.device)
            self.dst, self.accumulate = self._tmp, False

    def commit(self) -> None:
        p = self.p
        if self._tmp is not None:
            g = self._tmp.to(p.dtype)
            if p.grad is None:
                p.grad = g
            else:
                p.grad.add_(g)
        gradsink.mark_ready(p)


def _targets(*params):
    return [(_GradTarget(p) if (p is not None and p.requires_grad) else None) for p in params]


def _tp_world(group) -> int:
    return comm.get_world_size(group)


def _dgrad_all_reduce(dy: torch.Tensor, w: torch.Tensor, group) -> torch.Tensor:
    """``dy @ w`` summed over the tensor-parallel group (one fused kernel when tp > 1)."""
    if _tp_world(group) == 1:
        return G.linear_dgrad(dy, w)
    from ..parallel import collectives

    return collectives.dgrad_all_reduce(dy, w, group)


def _all_reduce_(t: torch.Tensor, group) -> torch.Tensor:
    """Sum ``t`` over the TP group in place with NCCL (fallback of the peer-memory kernels)."""
    if _tp_world(group) > 1:
        from ..parallel import collectives

        collectives.all_reduce_(t, group)
    return t


# ---------------------------------------------------------------------------
# Embedding
# ---------------------------------------------------------------------------


class _EmbeddingFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, ids, mod, wte, wpe):
        B, S = ids.shape
        emb = mod.wte
        group = emb.group
        tp = _tp_world(group)
        x = None
        if tp > 1:
            from ..parallel import collectives

            # Each row read from the rank that owns its vocabulary range (no reduction).
            x = collectives.embedding_tp(ids, wte, bf16_weight(wpe)[:S], group)
        if x is None:
            add_pos = tp == 1 or emb.rank == 0  # positions summed once across the TP reduction
            x = K.embedding_fwd(ids, bf16_weight(wte), bf16_weight(wpe)[:S] if add_pos else None, S,
                                vocab_start=emb.vocab_start if tp > 1 else 0)
            if tp > 1:
                _all_reduce_(x, group)
        ctx.mod, ctx.ids, ctx.shape = mod, ids, (B, S)
        return x.view(B, S, -1)

    @staticmethod
    def backward(ctx, dx):
        mod, ids = ctx.mod, ctx.ids
        B, S = ctx.shape
        dx2 = dx.reshape(B * S, -1)
        if dx2.stride(-1) != 1 or dx2.data_ptr() % 16 or dx2.stride(0) % 8:
            dx2 = dx2.contiguous()
        if dx2.dtype != torch.bfloat16:
            dx2 = dx2.to(torch.bfloat16)
        emb = mod.wte
        tw, tp_ = _targets(emb.weight, mod.wpe)
        if tp_ is not None:
            if S < tp_.dst.shape[0] and not tp_.accumulate:
                tp_.dst[S:].zero_()
            K.embedding_bwd_wpe(dx2, tp_.dst, B, S, accumulate=tp_.accumulate)
            tp_.commit()
        if tw is not None:
            if not tw.accumulate:
                tw.dst.zero_()
            K.embedding_bwd_wte(ids, dx2, tw.dst, vocab_start=emb.vocab_start if emb.world > 1 else 0)
            tw.commit()
        return None, None, None, None


def embedding_forward(mod, input_ids):
    return _EmbeddingFn.apply(input_ids, mod, mod.wte.weight, mod.wpe)


# ---------------------------------------------------------------------------
# Transformer block
# ---------------------------------------------------------------------------


def _as_bf16_2d(x: torch.Tensor) -> torch.Tensor:
    x2 = x.reshape(-1, x.shape[-1])
    if x2.dtype != torch.bfloat16:
        x2 = x2.to(torch.bfloat16)
    if x2.stride(-1) != 1 or x2.data_ptr() % 16 or x2.stride(0) % 8:
        x2 = x2.contiguous()
    return x2


class _BlockFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, blk, *params):
        B, S, C = x.shape
        xin = _as_bf16_2d(x)
        attn, mlp = blk.attn, blk.mlp
        group = blk.tp_group
        tp = _tp_world(group)
        H = attn.n_head_local
        D = attn.head_dim
        ln1g, ln1b, ln2g, ln2b, qkv_b, proj_b, fc_b, mproj_b = _fp32_params(
            blk.ln1.weight, blk.ln1.bias, blk.ln2.weight, blk.ln2.bias, attn.qkv.bias, attn.proj.bias,
            mlp.fc.bias, mlp.proj.bias)
        w_qkv, w_proj = bf16_weight(attn.qkv.weight), bf16_weight(attn.proj.weight)
        w_fc, w_mproj = bf16_weight(mlp.fc.weight), bf16_weight(mlp.proj.weight)

        h1, mu1, r1 = K.layernorm_fwd(xin, ln1g, ln1b, blk.ln1.eps)
        qkv = G.linear_fwd(h1, w_qkv, qkv_b)
        y, lse = K.attention_fwd(qkv, B, S, H, D)
        if tp == 1:
            x1 = G.linear_fwd(y, w_proj, proj_b, resid=xin)
        else:
            from ..parallel import collectives

            x1 = collectives.gemm_all_reduce(y, w_proj, proj_b, xin, group)
        h2, mu2, r2 = K.layernorm_fwd(x1, ln2g, ln2b, blk.ln2.eps)
        a, hpre = G.linear_fwd(h2, w_fc, fc_b, gelu=True)
        if tp == 1:
            x2 = G.linear_fwd(a, w_mproj, mproj_b, resid=x1)
        else:
            from ..parallel import collectives

            x2 = collectives.gemm_all_reduce(a, w_mproj, mproj_b, x1, group)

        ctx.blk = blk
        ctx.dims = (B, S, C, H, D, tp)
        ctx.saved = (xin, h1, mu1, r1, qkv, y, lse, x1, h2, mu2, r2, a, hpre, ln1g, ln2g)
        return x2.view(B, S, C)

    @staticmethod
    def backward(ctx, dx2):
        blk = ctx.blk
        B, S, C, H, D, tp = ctx.dims
        xin, h1, mu1, r1, qkv, y, lse, x1, h2, mu2, r2, a, hpre, ln1g, ln2g = ctx.saved
        ctx.saved = None
        attn, mlp = blk.attn, blk.mlp
        group = blk.tp_group
        dx2 = _as_bf16_2d(dx2)
        w_qkv, w_proj = bf16_weight(attn.qkv.weight), bf16_weight(attn.proj.weight)
        w_fc, w_mproj = bf16_weight(mlp.fc.weight), bf16_weight(mlp.proj.weight)

        # MLP projection (row-parallel): weight grad, then d(pre-activation) with GELU' fused.
        (t_mw,) = _targets(mlp.proj.weight)
        if t_mw is not None:
            G.linear_wgrad(dx2, a, t_mw.dst, accumulate=t_mw.accumulate)
            t_mw.commit()
        # MLP fc (column-parallel); its bias gradient's first stage comes out of the
        # dGELU epilogue (per-32-row column sums), so dh is not read back for it.
        t_fw, t_fb = _targets(mlp.fc.weight, mlp.fc.bias)
        fb_part = None
        if t_fb is not None:
            fb_part = torch.empty(-(-dx2.shape[0] // 32) * w_mproj.shape[1], dtype=torch.float32,
                                  device=dx2.device)
        dh = G.linear_dgrad(dx2, w_mproj, gelu_preact=hpre, colsum_partial=fb_part)
        if t_fw is not None:
            G.linear_wgrad(dh, h2, t_fw.dst, accumulate=t_fw.accumulate)
            t_fw.commit()
        if t_fb is not None:
            K.colsum_final(fb_part, -(-dx2.shape[0] // 32), t_fb.dst, accumulate=t_fb.accumulate)
            t_fb.commit()
        dh2 = _dgrad_all_reduce(dh, w_fc, group)  # f: gradient of the replicated LN2 output
        # LN2 backward + residual, with both row-parallel bias gradients fused.
        t_l2g, t_l2b, t_mb, t_pb = _targets(blk.ln2.weight, blk.ln2.bias, mlp.proj.bias, attn.proj.bias)
        dx1 = K.layernorm_bwd(
            dh2, x1, mu2, r2, ln2g, resid_grad=dx2,
            dgamma=t_l2g.dst if t_l2g else None, acc_gamma=bool(t_l2g and t_l2g.accumulate),
            dbeta=t_l2b.dst if t_l2b else None, acc_beta=bool(t_l2b and t_l2b.accumulate),
            colsum_resid=t_mb.dst if t_mb else None, acc_resid=bool(t_mb and t_mb.accumulate),
            colsum_out=t_pb.dst if t_pb else None, acc_out=bool(t_pb and t_pb.accumulate))
        for t in (t_mb, t_l2g, t_l2b, t_pb):
            if t is not None:
                t.commit()
        # Attention output projection (row-parallel)
        (t_pw,) = _targets(attn.proj.weight)
        if t_pw is not None:
            G.linear_wgrad(dx1, y, t_pw.dst, accumulate=t_pw.accumulate)
            t_pw.commit()
        # dO, with the attention backward's delta = rowsum(dO * O) from the same epilogue.
        delta = None
        if D == 64 and K.attention_bwd_impl() == "tc":
            delta = torch.empty(B * H * S, dtype=torch.float32, device=dx1.device)
            dy = G.linear_dgrad(dx1, w_proj, dot=(y, delta, D, S))
        else:
            dy = G.linear_dgrad(dx1, w_proj)
        dqkv = K.attention_bwd(qkv, y, dy, lse, B, S, H, D, delta=delta)
        # QKV (column-parallel)
        t_qw, t_qb = _targets(attn.qkv.weight, attn.qkv.bias)
        if t_qw is not None:
            G.linear_wgrad(dqkv, h1, t_qw.dst, accumulate=t_qw.accumulate)
            t_qw.commit()
        if t_qb is not None:
            K.colsum(dqkv, t_qb.dst, accumulate=t_qb.accumulate)
            t_qb.commit()
        dh1 = _dgrad_all_reduce(dqkv, w_qkv, group)
        t_l1g, t_l1b = _targets(blk.ln1.weight, blk.ln1.bias)
        dx = K.layernorm_bwd(
            dh1, xin, mu1, r1, ln1g, resid_grad=dx1,
            dgamma=t_l1g.dst if t_l1g else None, acc_gamma=bool(t_l1g and t_l1g.accumulate),
            dbeta=t_l1b.dst if t_l1b else None, acc_beta=bool(t_l1b and t_l1b.accumulate))
        for t in (t_l1g, t_l1b):
            if t is not None:
                t.commit()
        return (dx.view(B, S, C), None) + (None,) * len(_block_params(blk))


def _block_params(blk):
    return [p for p in blk.parameters()]


def block_forward(blk, x):
    if x.dim() != 3:
        raise ValueError("fused block expects [batch, seq, hidden] input")
    return _BlockFn.apply(x, blk, *_block_params(blk))


# ---------------------------------------------------------------------------
# LM head: final LayerNorm + (vocabulary-sharded) projection [+ cross-entropy]
# ---------------------------------------------------------------------------


def _ce_stats_tp(tmax, tsum, tgt, group):
    """Per-row (max, sumexp, target logit) combined over the TP group -> (lse, loss_rows).

    One peer-memory kernel (md_ce_tp) on a single node; otherwise an all_reduce(MAX) and a
    packed all_reduce(SUM) over NCCL (tensor_parallel.py:457-474)."""
    from ..parallel import collectives

    if _tp_world(group) > 1:
        fused = collectives.ce_tp_stats(tmax, tsum, tgt, group)
        if fused is not None:
            return fused
    rmax, rsum, _, _ = K.ce_stats(tmax, tsum, finish=False)
    if _tp_world(group) > 1:
        gmax = rmax.clone()
        comm.all_reduce(gmax, op=torch.distributed.ReduceOp.MAX, group=group)
        packed = torch.stack([rsum * torch.exp(rmax - gmax), tgt])
        comm.all_reduce(packed, group=group)
        rsum, tgt, rmax = packed[0], packed[1], gmax
    lse = rmax + torch.log(rsum)
    return lse, lse - tgt


class _HeadFn(torch.autograd.Function):
    """LayerNorm -> logits GEMM, with the cross-entropy fused when ``targets`` is given."""

    @staticmethod
    def forward(ctx, x, head, targets, ln_w, ln_b, w):
        B, S, C = x.shape
        # An unused output (usually the logits) must arrive as None, not as a
        # materialised zero tensor of [tokens, vocab] that would then be added.
        ctx.set_materialize_grads(False)
        xin = _as_bf16_2d(x)
        lnw, lnb = fp32_param(head.ln_f.weight), fp32_param(head.ln_f.bias)
        h, mu, r = K.layernorm_fwd(xin, lnw, lnb, head.ln_f.eps)
        wb = bf16_weight(head.head.weight)
        V = wb.shape[0]
        M = B * S
        group = head.tp_group
        logits = G.empty_padded(M, V, device=x.device)
        ctx.has_loss = targets is not None
        if targets is None:
            G.linear_fwd(h, wb, out=logits)
            loss = None
        else:
            tgt_flat = targets.reshape(-1).contiguous()
            tiles = -(-V // G.CE_SLAB)
            tmax = torch.empty(tiles, M, dtype=torch.float32, device=x.device)
            tsum = torch.empty_like(tmax)
            ttgt = torch.zeros(M, dtype=torch.float32, device=x.device)
            col0 = head.vocab_start if _tp_world(group) > 1 else 0
            G.gemm(h, wb, logits, M=M, N=V, K=C, lda=h.stride(0), ldb=wb.stride(0), ldd=logits.stride(0),
                   epi=G.EPI_CE, ce=(tgt_flat, tmax, tsum, ttgt), ce_col_offset=col0)
            if _tp_world(group) == 1:
                _, _, lse, loss_rows = K.ce_stats(tmax, tsum, ttgt, finish=True)
            else:
                lse, loss_rows = _ce_stats_tp(tmax, tsum, ttgt, group)
            loss = loss_rows.mean()
            ctx.lse, ctx.targets, ctx.col0 = lse, tgt_flat, col0
        ctx.head = head
        ctx.dims = (B, S, C, V)
        ctx.saved = (xin, h, mu, r, lnw, logits)
        out_logits = logits.view(B, S, V)
        if loss is None:
            return out_logits, torch.zeros((), device=x.device)
        return out_logits, loss

    @staticmethod
    def backward(ctx, g_logits, g_loss):
        head = ctx.head
        B, S, C, V = ctx.dims
        M = B * S
        xin, h, mu, r, lnw, logits = ctx.saved
        ctx.saved = None
        group = head.tp_group
        if ctx.has_loss and g_loss is not None:
            dlogits = K.ce_backward(logits, ctx.lse, ctx.targets, g_loss.float().reshape(1), 1.0 / M, V,
                                    col_offset=ctx.col0)
            if g_logits is not None:
                dlogits += g_logits.reshape(M, V).to(dlogits.dtype)
        elif g_logits is not None:
            dlogits = _as_bf16_2d(g_logits.reshape(M, V))
        else:
            return None, None, None, None, None, None
        wb = bf16_weight(head.head.weight)
        (t_w,) = _targets(head.head.weight)
        if t_w is not None:
            G.linear_wgrad(dlogits, h, t_w.dst, accumulate=t_w.accumulate)
            t_w.commit()
        dh = _dgrad_all_reduce(dlogits, wb, group)  # f backward of the column-parallel head
        t_g, t_b = _targets(head.ln_f.weight, head.ln_f.bias)
        dx = K.layernorm_bwd(dh, xin, mu, r, lnw,
                             dgamma=t_g.dst if t_g else None, acc_gamma=bool(t_g and t_g.accumulate),
                             dbeta=t_b.dst if t_b else None, acc_beta=bool(t_b and t_b.accumulate))
        for t in (t_g, t_b):
            if t is not None:
                t.commit()
        return dx.view(B, S, C), None, None, None, None, None


def head_logits(head, x):
    logits, _ = _HeadFn.apply(x, head, None, head.ln_f.weight, head.ln_f.bias, head.head.weight)
    return logits


def head_logits_and_loss(head, x, targets):
    return _HeadFn.apply(x, head, targets, head.ln_f.weight, head.ln_f.bias, head.head.weight)


def head_loss(head, x, targets):
    return head_logits_and_loss(head, x, targets)[1]
