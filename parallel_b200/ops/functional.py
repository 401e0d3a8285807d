"""Differentiable fused ops of the Qwen3 / Qwen3-MoE blocks.

Every op has two implementations behind one call:

* CUDA tensors run the sm_100a kernels (``parallel_b200._C``) inside a
  ``torch.autograd.Function`` whose backward is also made of kernels;
* CPU tensors run the plain PyTorch statement of the same math (fp32 in the
  CPU tests), which is the numerics oracle and the gloo/CPU training path.

Numerics follow the HF modules the reference trains (transformers Qwen3 /
Qwen3-MoE modeling files, loaded by parallel/parallel/engine/
model_loading.py:17-35): RMSNorm in fp32 with the normalised value rounded to
the input dtype before the weight multiply; rotate-half RoPE; causal GQA
attention with softmax scale 1/sqrt(head_dim); SwiGLU MLP; mean token
cross-entropy over labels != -100.
"""
from __future__ import annotations

import math
import os

import torch
import torch.nn.functional as F

from ._ext import ext
from . import gemm as G

IGNORE_INDEX = -100


# ----------------------------------------------------------------- helpers
def fused_rows(*ws: torch.Tensor) -> torch.Tensor:
    """Row-concatenation of 2-D weights; a zero-copy view when they are
    adjacent in one storage (FSDP buckets and the model allocator lay q/k/v
    and gate/up out that way), else a copy."""
    w0 = ws[0]
    ok = all(w.dim() == 2 and w.is_contiguous() and w.dtype == w0.dtype and w.shape[1] == w0.shape[1]
             for w in ws)
    if ok:
        try:
            same = all(w.untyped_storage().data_ptr() == w0.untyped_storage().data_ptr() for w in ws)
        except Exception:
            same = False
        if same:
            es = w0.element_size()
            for a, b in zip(ws[:-1], ws[1:]):
                if b.data_ptr() != a.data_ptr() + a.numel() * es:
                    same = False
                    break
        if same:
            rows = sum(w.shape[0] for w in ws)
            return w0.as_strided((rows, w0.shape[1]), (w0.shape[1], 1))
    return torch.cat(ws, 0)


def _split_rows(t: torch.Tensor, sizes) -> list[torch.Tensor]:
    out, r = [], 0
    for s in sizes:
        out.append(t[r:r + s])
        r += s
    return out


_ROPE_CACHE: dict = {}


def rope_tables(inv_freq: torch.Tensor, S: int, dtype: torch.dtype, device: torch.device,
                attention_scaling: float = 1.0):
    """HF default RoPE: cos/sin of pos * inv_freq (fp32), duplicated halves,
    cast to the activation dtype.  Cached per (S, dtype, device, inv_freq)."""
    key = (S, dtype, str(device), inv_freq.data_ptr(), inv_freq._version)
    hit = _ROPE_CACHE.get(key)
    if hit is not None:
        return hit
    with torch.autocast(device_type=device.type, enabled=False):
        pos = torch.arange(S, device=device, dtype=torch.float32)
        freqs = pos[:, None] * inv_freq.to(device=device, dtype=torch.float32)[None, :]
        emb = torch.cat((freqs, freqs), dim=-1)
        cos = (emb.cos() * attention_scaling).to(dtype).contiguous()
        sin = (emb.sin() * attention_scaling).to(dtype).contiguous()
    if len(_ROPE_CACHE) > 16:
        _ROPE_CACHE.clear()
    _ROPE_CACHE[key] = (cos, sin)
    return cos, sin


def _rms_ref(x: torch.Tensor, w: torch.Tensor, eps: float) -> torch.Tensor:
    dt = x.dtype
    xf = x.to(torch.float32)
    xf = xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + eps)
    return w * xf.to(dt)


def _rotate_half(x):
    h = x.shape[-1] // 2
    return torch.cat((-x[..., h:], x[..., :h]), dim=-1)


# ----------------------------------------------------------------- RMSNorm
class _RMSNormFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, w, eps):
        shape = x.shape
        x2 = x.reshape(-1, shape[-1])
        if not x2.is_contiguous():
            x2 = x2.contiguous()
        y = torch.empty_like(x2)
        rstd = torch.empty(x2.shape[0], device=x.device, dtype=torch.float32)
        ext().rmsnorm_fwd(x2, w, y, rstd, eps)
        ctx.save_for_backward(x2, w, rstd)
        ctx.shape = shape
        return y.view(shape)

    @staticmethod
    def backward(ctx, dy):
        x2, w, rstd = ctx.saved_tensors
        dy2 = dy.reshape(-1, x2.shape[1])
        if not dy2.is_contiguous():
            dy2 = dy2.contiguous()
        dx = torch.empty_like(x2)
        # the kernel writes block partials and sums them in a fixed order into dw
        dw = torch.empty(x2.shape[1], device=x2.device, dtype=w.dtype)
        ext().rmsnorm_bwd(dy2, x2, w, rstd, dx, dw)
        return dx.view(ctx.shape), dw, None


def rms_norm(x: torch.Tensor, w: torch.Tensor, eps: float) -> torch.Tensor:
    if x.is_cuda:
        return _RMSNormFn.apply(x, w, eps)
    return _rms_ref(x, w, eps)


class _ResidualRMSNormFn(torch.autograd.Function):
    """(x, norm(x)) for a residual stream that feeds both a norm and a later
    residual add; the backward sums both gradients inside the norm kernel."""

    @staticmethod
    def forward(ctx, x, w, eps):
        shape = x.shape
        x2 = x.reshape(-1, shape[-1])
        if not x2.is_contiguous():
            x2 = x2.contiguous()
        y = torch.empty_like(x2)
        rstd = torch.empty(x2.shape[0], device=x.device, dtype=torch.float32)
        ext().rmsnorm_fwd(x2, w, y, rstd, eps)
        ctx.save_for_backward(x2, w, rstd)
        ctx.shape = shape
        return x.view_as(x), y.view(shape)

    @staticmethod
    def backward(ctx, dres, dy):
        x2, w, rstd = ctx.saved_tensors
        H = x2.shape[1]
        dx = torch.empty_like(x2)
        dw = torch.empty(H, device=x2.device, dtype=w.dtype)
        if dy is None:
            return dres, None, None
        dy2 = dy.reshape(-1, H)
        if not dy2.is_contiguous():
            dy2 = dy2.contiguous()
        r2 = None
        if dres is not None:
            r2 = dres.reshape(-1, H)
            if not r2.is_contiguous():
                r2 = r2.contiguous()
        ext().rmsnorm_bwd(dy2, x2, w, rstd, dx, dw, r2)
        return dx.view(ctx.shape), dw, None


def residual_rms_norm(x: torch.Tensor, w: torch.Tensor, eps: float):
    """Returns (x, norm(x)); use the first output for the residual add."""
    if x.is_cuda:
        return _ResidualRMSNormFn.apply(x, w, eps)
    return x, _rms_ref(x, w, eps)


# ----------------------------------------------------------------- attention block
# Upper bound of the attention backward's dS tile buffer (bf16, causal tiles of
# every head); larger problems use the fp32 dQ accumulator instead.
_ATTN_DS_LIMIT_BYTES = int(os.environ.get("PB_ATTN_DS_LIMIT_BYTES", str(4 << 30)))


class _AttentionFn(torch.autograd.Function):
    """qkv = h W_qkv^T -> per-head q/k RMSNorm + RoPE -> causal GQA flash
    attention.  Returns the attention output [T, nq*D] (before o_proj)."""

    @staticmethod
    def forward(ctx, h, wq, wk, wv, qw, kw, cos, sin, B, S, nq, nkv, D, eps, stash=None, sp=None):
        T = B * S
        wqkv = fused_rows(wq, wk, wv)
        ctx.sp = sp
        ctx.h_shape = h.shape
        if sp is not None:
            # sequence parallel: h is this rank's [B*S/tp, H] shard; the gather
            # runs inside the QKV GEMM and the gathered rows are kept for dW
            h_local = h.reshape(-1, h.shape[-1])
            qkv, h = sp.all_gather_gemm(h_local if h_local.is_contiguous() else h_local.contiguous(), wqkv, B, S)
        else:
            qkv = G.linear(h.reshape(T, -1), wqkv)
        q = torch.empty(T, nq * D, device=h.device, dtype=h.dtype)
        k = torch.empty(T, nkv * D, device=h.device, dtype=h.dtype)
        rstd = torch.empty(T, nq + nkv, device=h.device, dtype=torch.float32)
        ext().qknorm_rope_fwd(qkv, qw, kw, cos, sin, q, k, rstd, S, nq, nkv, eps)
        v = qkv[:, (nq + nkv) * D:]
        if stash is not None and stash.get("mode") == "reuse" and "o" in stash:
            # activation-checkpoint recompute: the attention output and its
            # log-sum-exp were kept from the forward pass (same inputs, same result)
            o, lse = stash.pop("o"), stash.pop("lse")
        else:
            o = torch.empty(T, nq * D, device=h.device, dtype=h.dtype)
            lse = torch.zeros(B * nq * S + 128, device=h.device, dtype=torch.float32)
            ext().attn_fwd(q, k, v, o, lse, B, S, nq, nkv, 1.0 / math.sqrt(D), True)
            if stash is not None and stash.get("mode") == "save":
                stash["o"], stash["lse"] = o, lse
        ctx.save_for_backward(h, wq, wk, wv, qw, kw, cos, sin, qkv, q, k, o, lse, rstd)
        ctx.dims = (B, S, nq, nkv, D)
        return o

    @staticmethod
    def backward(ctx, do):
        h, wq, wk, wv, qw, kw, cos, sin, qkv, q, k, o, lse, rstd = ctx.saved_tensors
        B, S, nq, nkv, D = ctx.dims
        T = B * S
        do = do if do.is_contiguous() else do.contiguous()
        dqkv = torch.empty_like(qkv)
        dq = torch.empty_like(q)
        dk = torch.empty_like(k)
        dv = dqkv[:, (nq + nkv) * D:]
        v = qkv[:, (nq + nkv) * D:]
        delta = torch.empty(2 * (B * nq * S + 128), device=h.device, dtype=torch.float32)
        ds_elems = ext().attn_bwd_ds_elems(B, S, nq, True)
        if ds_elems * 2 <= _ATTN_DS_LIMIT_BYTES:
            # dS tiles stored once, dQ from a second tcgen05 kernel (no fp32 accumulator)
            ds_buf = torch.empty(ds_elems, device=h.device, dtype=torch.bfloat16)
            dq_acc = torch.empty(0, device=h.device, dtype=torch.float32)
        else:  # very long sequences: dQ reduced into an fp32 accumulator in place
            ds_buf = None
            dq_acc = torch.empty(T, nq * D, device=h.device, dtype=torch.float32)
        ext().attn_bwd(q, k, v, o, do, lse, delta, dq_acc, dq, dk, dv, B, S, nq, nkv, 1.0 / math.sqrt(D), True,
                       None, ds_buf)
        dqw = torch.empty(D, device=h.device, dtype=qw.dtype)
        dkw = torch.empty(D, device=h.device, dtype=kw.dtype)
        ext().qknorm_rope_bwd(dq, dk, qkv, qw, kw, cos, sin, rstd, dqkv, dqw, dkw, S, nq, nkv)
        wqkv = fused_rows(wq, wk, wv)
        h2 = h.reshape(T, -1)
        if ctx.sp is not None:
            dh = ctx.sp.gemm_reduce_scatter(dqkv, wqkv, B, S, b_mn=True).view(ctx.h_shape)
        else:
            dh = G.linear_dgrad(dqkv, wqkv).view(h.shape)
        dw = G.linear_wgrad(dqkv, h2)
        gq, gk, gv = _split_rows(dw, (wq.shape[0], wk.shape[0], wv.shape[0]))
        return dh, gq, gk, gv, dqw, dkw, None, None, None, None, None, None, None, None, None, None


def attention_block(h, wq, wk, wv, q_norm_w, k_norm_w, inv_freq, B, S, nq, nkv, D, eps, stash=None, sp=None):
    """Self-attention up to (not including) o_proj: returns [B*S, nq*D].

    ``stash`` (CUDA path): a dict with mode "save" keeps the attention output
    and log-sum-exp; mode "reuse" consumes them instead of recomputing the
    attention kernel (selective recompute under activation checkpointing)."""
    if h.is_cuda:
        cos, sin = rope_tables(inv_freq, S, h.dtype, h.device)
        return _AttentionFn.apply(h, wq, wk, wv, q_norm_w, k_norm_w, cos, sin, B, S, nq, nkv, D, eps, stash, sp)
    cos, sin = rope_tables(inv_freq, S, h.dtype, h.device)
    x = h.reshape(B, S, -1)
    q = F.linear(x, wq).view(B, S, nq, D)
    k = F.linear(x, wk).view(B, S, nkv, D)
    v = F.linear(x, wv).view(B, S, nkv, D)
    q = _rms_ref(q, q_norm_w, eps).transpose(1, 2)
    k = _rms_ref(k, k_norm_w, eps).transpose(1, 2)
    v = v.transpose(1, 2)
    c, s = cos[None, None], sin[None, None]
    q = q * c + _rotate_half(q) * s
    k = k * c + _rotate_half(k) * s
    if nq != nkv:
        k = k.repeat_interleave(nq // nkv, dim=1)
        v = v.repeat_interleave(nq // nkv, dim=1)
    o = F.scaled_dot_product_attention(q, k, v, is_causal=True, scale=1.0 / math.sqrt(D))
    return o.transpose(1, 2).reshape(B * S, nq * D)


# ----------------------------------------------------------------- linear (+ residual)
class _LinearFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, w, residual):
        x2 = x.reshape(-1, x.shape[-1])
        if not x2.is_contiguous():
            x2 = x2.contiguous()
        r2 = None if residual is None else residual.reshape(-1, w.shape[0])
        y = G.linear(x2, w, residual=r2)
        ctx.save_for_backward(x2, w)
        ctx.has_res = residual is not None
        ctx.in_shape = x.shape
        out_shape = residual.shape if residual is not None else (*x.shape[:-1], w.shape[0])
        return y.view(out_shape)

    @staticmethod
    def backward(ctx, dy):
        x2, w = ctx.saved_tensors
        dy2 = dy.reshape(-1, w.shape[0])
        if not dy2.is_contiguous():
            dy2 = dy2.contiguous()
        dx = G.linear_dgrad(dy2, w).view(ctx.in_shape)
        dw = G.linear_wgrad(dy2, x2)
        return dx, dw, (dy if ctx.has_res else None)


def linear(x: torch.Tensor, w: torch.Tensor, residual: torch.Tensor | None = None) -> torch.Tensor:
    """``residual + x @ w.T`` (residual optional)."""
    if x.is_cuda:
        return _LinearFn.apply(x, w, residual)
    y = F.linear(x, w)
    if residual is not None:
        y = residual + y.view(residual.shape)
    return y


# ----------------------------------------------------------------- SwiGLU MLP
class _MLPFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, wg, wu, wd, residual, output_unused=False):
        I = wg.shape[0]
        x2 = x.reshape(-1, x.shape[-1])
        if not x2.is_contiguous():
            x2 = x2.contiguous()
        wgu = fused_rows(wg, wu)
        h, gu = G.linear_swiglu(x2, wgu, I)
        r2 = None if residual is None else residual.reshape(-1, wd.shape[0])
        if output_unused:
            # activation-checkpoint recompute: only the saved tensors matter (the
            # backward of the down projection needs h and its weight, not its
            # output), so the down GEMM is not run and the output is left unset
            out = torch.empty(x2.shape[0], wd.shape[0], device=x.device, dtype=x.dtype)
        else:
            out = G.linear(h, wd, residual=r2)
        ctx.save_for_backward(x2, wg, wu, wd, gu, h)
        ctx.has_res = residual is not None
        ctx.in_shape = x.shape
        return out.view(*x.shape[:-1], wd.shape[0])

    @staticmethod
    def backward(ctx, dy):
        x2, wg, wu, wd, gu, h = ctx.saved_tensors
        I = wg.shape[0]
        dy2 = dy.reshape(-1, wd.shape[0])
        if not dy2.is_contiguous():
            dy2 = dy2.contiguous()
        dh = G.linear_dgrad(dy2, wd)
        dwd = G.linear_wgrad(dy2, h)
        dgu = torch.empty_like(gu)
        ext().swiglu_bwd(dh, gu, dgu)
        wgu = fused_rows(wg, wu)
        dx = G.linear_dgrad(dgu, wgu).view(ctx.in_shape)
        dwgu = G.linear_wgrad(dgu, x2)
        return dx, dwgu[:I], dwgu[I:], dwd, (dy if ctx.has_res else None), None


def swiglu_mlp(x, wg, wu, wd, residual=None, output_unused: bool = False):
    """``residual + down(silu(gate x) * up x)``.  ``output_unused`` (CUDA): the
    caller only differentiates through the result (an activation-checkpoint
    recompute), so its value is not computed; gradients are unchanged."""
    if x.is_cuda:
        return _MLPFn.apply(x, wg, wu, wd, residual, output_unused)
    y = F.linear(F.silu(F.linear(x, wg)) * F.linear(x, wu), wd)
    if residual is not None:
        y = residual + y
    return y


# ----------------------------------------------------------------- embedding
class TiedGrad:
    """Hand-off between the LM head and the embedding of one forward pass when
    they share a weight: the LM head's backward leaves its (dense) weight
    gradient here, and the embedding's backward - which autograd runs later,
    before it sums the two contributions - adds its few touched rows into that
    tensor in place and returns no gradient of its own.  This replaces a
    full-vocabulary fp32 accumulator, its cast and a dense bf16 add
    (~2 GB of traffic at a 151,936-token vocabulary) with a row update."""

    __slots__ = ("grad", "w_head", "w_emb")

    def __init__(self):
        self.grad = None
        self.w_head = None
        self.w_emb = None


class _EmbeddingFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, ids, w, v0, tied, reader):
        flat = ids.reshape(-1)
        if not flat.is_contiguous():
            flat = flat.contiguous()
        if reader is not None:
            # rows fetched by the caller's reader (FSDP: from the peers' row shards)
            out = reader(flat)
        else:
            out = torch.empty(flat.numel(), w.shape[1], device=w.device, dtype=w.dtype)
            ext().embedding_fwd(flat, w, out, v0)
        ctx.save_for_backward(flat)
        ctx.v0 = v0
        ctx.wshape = w.shape
        ctx.wdtype = w.dtype
        ctx.tied = tied
        if tied is not None:
            tied.w_emb = w
        return out.view(*ids.shape, w.shape[1])

    @staticmethod
    def backward(ctx, dy):
        (flat,) = ctx.saved_tensors
        dy2 = dy.reshape(-1, ctx.wshape[1])
        if not dy2.is_contiguous() or dy2.dtype != torch.bfloat16:
            dy2 = dy2.contiguous().to(torch.bfloat16)
        sid, perm = torch.sort(flat, stable=True)
        tied, ctx.tied = ctx.tied, None
        pending = None
        if tied is not None:
            pending, tied.grad = tied.grad, None
            if not (tied.w_head is tied.w_emb and pending is not None and pending.shape == ctx.wshape
                    and pending.dtype == torch.bfloat16 and pending.is_contiguous()):
                pending = None
        if pending is not None:
            ext().embedding_bwd(sid, perm, dy2, pending, ctx.v0, True)
            return None, None, None, None, None
        gb = torch.zeros(ctx.wshape, device=dy.device, dtype=torch.bfloat16)
        ext().embedding_bwd(sid, perm, dy2, gb, ctx.v0, False)
        return None, gb.to(ctx.wdtype), None, None, None


def embedding(ids: torch.Tensor, w: torch.Tensor, vocab_start: int = 0, tied: TiedGrad | None = None,
              reader=None) -> torch.Tensor:
    """Rows of ``w`` for ids in [vocab_start, vocab_start + len(w)), zeros elsewhere.
    ``reader(flat_ids) -> rows`` (CUDA only) supplies the forward rows instead
    of ``w``; the gradient still goes to ``w``."""
    if w.is_cuda:
        return _EmbeddingFn.apply(ids, w, vocab_start, tied, reader)
    if vocab_start == 0 and (ids.numel() == 0 or int(ids.max()) < w.shape[0]):
        return F.embedding(ids, w)
    local = ids - vocab_start
    mask = (local < 0) | (local >= w.shape[0])
    out = F.embedding(local.masked_fill(mask, 0), w)
    return out.masked_fill(mask[..., None], 0)


# ----------------------------------------------------------------- LM head + CE
class _LMHeadCEFn(torch.autograd.Function):
    """Mean cross-entropy of ``h @ W.T`` against ``labels``; the gradient is
    computed in the forward pass (one pass over each logits block, no fp32
    logits ever materialised) and scaled by the incoming grad in backward."""

    @staticmethod
    def forward(ctx, h, w, labels, max_block_bytes, tied):
        T, H = h.shape
        V = w.shape[0]
        labels = labels.reshape(-1).contiguous()
        # 1 / #valid labels, per-row (lse, target logit), and the mean loss
        # summed over the rows in a fixed order: a few kernels, no atomics
        inv = torch.empty(1, device=h.device, dtype=torch.float32)
        ext().ce_valid_inv(labels, inv)
        lse = torch.empty(T, device=h.device, dtype=torch.float32)
        tgt = torch.empty(T, device=h.device, dtype=torch.float32)
        loss = torch.empty(1, device=h.device, dtype=torch.float32)
        rows = max(128, min(T, int(max_block_bytes // (V * 2)) // 128 * 128))
        dh = torch.empty_like(h)
        single = rows >= T
        dw = None if single else torch.empty(V, H, device=h.device, dtype=torch.float32)
        for r0 in range(0, T, rows):
            r1 = min(T, r0 + rows)
            hb = h[r0:r1]
            logits = G.linear(hb, w)
            ext().ce_fwd_bwd(logits, labels[r0:r1], 0, inv, lse[r0:r1], False, tgt[r0:r1], True)
            G.linear_dgrad(logits, w, out=dh[r0:r1])
            if single:
                dw = G.linear_wgrad(logits, hb)
            else:
                G.linear_wgrad(logits, hb, out=dw, accumulate=r0 > 0)
            del logits
        ext().ce_loss_reduce(lse, tgt, labels, inv, loss, False)
        if not single:
            dwb = torch.empty(V, H, device=h.device, dtype=w.dtype)
            ext().cast_f32_to_bf16(dw, dwb)
            dw = dwb
        ctx.save_for_backward(dh, dw)
        ctx.tied = tied
        if tied is not None:
            tied.w_head = w
        return loss.reshape(())

    @staticmethod
    def backward(ctx, g):
        # the saved gradients are scaled (and, when tied, completed by the
        # embedding backward) in place: one backward pass per forward
        if getattr(ctx, "consumed", False):
            raise RuntimeError("lm_head_cross_entropy supports one backward pass per forward")
        ctx.consumed = True
        dh, dw = ctx.saved_tensors
        g = g.reshape(1).to(torch.float32)
        if dh.dtype == torch.bfloat16 and dw.dtype == torch.bfloat16 and dh.is_contiguous() and dw.is_contiguous():
            # scale in place (a no-op kernel when the incoming gradient is 1)
            ext().scale_by_scalar(dh, g)
            ext().scale_by_scalar(dw, g)
        else:
            dh, dw = dh * g.to(dh.dtype), dw * g.to(dw.dtype)
        if ctx.tied is not None:
            ctx.tied.grad = dw
            ctx.tied = None
        return dh, dw, None, None, None


def lm_head_cross_entropy(h: torch.Tensor, w: torch.Tensor, labels: torch.Tensor,
                          max_block_bytes: int = 6 << 30, tied: TiedGrad | None = None) -> torch.Tensor:
    """Mean CE over labels != -100 of logits = h @ w.T; h [T, H], labels [T].
    ``tied`` (shared with the embedding call of the same pass when the two
    share ``w``) lets the embedding backward update this gradient in place."""
    h2 = h.reshape(-1, h.shape[-1])
    if h2.is_cuda:
        if not h2.is_contiguous():
            h2 = h2.contiguous()
        return _LMHeadCEFn.apply(h2, w, labels, max_block_bytes, tied)
    logits = F.linear(h2, w).float()
    return F.cross_entropy(logits, labels.reshape(-1), ignore_index=IGNORE_INDEX)


def shift_labels(labels: torch.Tensor) -> torch.Tensor:
    """HF causal-LM convention: position t is scored against labels[t+1]."""
    out = torch.full_like(labels, IGNORE_INDEX)
    out[..., :-1] = labels[..., 1:]
    return out
