"""Vocabulary-parallel cross-entropy (logits sharded over the TP group).

Numerics of ``F.cross_entropy`` under DTensor ``loss_parallel`` (the
reference, parallel/parallel/engine/model_parallel/loss_parallel.py:22-69):
fp32 log-sum-exp merged across ranks by max / sum-exp all-reduces, the
target logit contributed by its owning rank, mean over labels != -100.

Two entry points:
* ``vocab_parallel_cross_entropy(local_logits, labels, tp_mesh, vocab_size)``
  - the reference API, over materialised local logits;
* ``vocab_parallel_lm_head_ce(h, w_local, labels, group, vocab_start)`` -
  the B200 path: LM-head GEMM blocks + CE kernels, global statistics merged
  per block, gradients produced in the forward pass; full-vocabulary logits
  are never formed and local logits only one row block at a time.
"""
from __future__ import annotations

from contextlib import nullcontext

import torch
import torch.distributed as dist

from ...ops import gemm as G
from ...ops._ext import ext
from ...profiling import collective_profile

IGNORE = -100


def loss_parallel_context(enabled: bool):
    """The backward needs no special context here (kept for API parity)."""
    return nullcontext()


class _VocabParallelCE(torch.autograd.Function):
    @staticmethod
    def forward(ctx, logits, labels, group, vocab_start, reduction):
        lf = logits.float()
        T, V = lf.shape
        m = lf.max(dim=-1).values
        with collective_profile("tp_all_reduce", value=m, mode="loss_parallel", detail="max"):
            dist.all_reduce(m, op=dist.ReduceOp.MAX, group=group)
        e = torch.exp(lf - m[:, None])
        s = e.sum(-1)
        with collective_profile("tp_all_reduce", value=s, mode="loss_parallel", detail="sumexp"):
            dist.all_reduce(s, op=dist.ReduceOp.SUM, group=group)
        lse = m + torch.log(s)
        local = labels - vocab_start
        inside = (labels != IGNORE) & (local >= 0) & (local < V)
        tgt = torch.zeros(T, dtype=torch.float32, device=lf.device)
        idx = local.clamp(0, V - 1)
        tgt = torch.where(inside, lf.gather(1, idx[:, None])[:, 0], tgt)
        with collective_profile("tp_all_reduce", value=tgt, mode="loss_parallel", detail="target"):
            dist.all_reduce(tgt, op=dist.ReduceOp.SUM, group=group)
        valid = labels != IGNORE
        per = torch.where(valid, lse - tgt, torch.zeros_like(lse))
        n = valid.sum()
        if reduction == "mean":
            out = per.sum() / n.clamp_min(1)
        elif reduction == "sum":
            out = per.sum()
        else:
            out = per
        ctx.save_for_backward(e, s, idx, inside, valid, n)
        ctx.reduction, ctx.in_dtype = reduction, logits.dtype
        return out

    @staticmethod
    def backward(ctx, g):
        e, s, idx, inside, valid, n = ctx.saved_tensors
        grad = e / s[:, None]
        grad[torch.arange(grad.shape[0], device=grad.device)[inside], idx[inside]] -= 1.0
        grad = grad * valid[:, None]
        if ctx.reduction == "mean":
            grad = grad * (g / n.clamp_min(1))
        elif ctx.reduction == "sum":
            grad = grad * g
        else:
            grad = grad * g[:, None]
        return grad.to(ctx.in_dtype), None, None, None, None


def vocab_parallel_cross_entropy(local_logits, labels, *, tp_mesh, vocab_size: int, reduction: str = "mean"):
    """CE of vocab-sharded logits ``[..., V/tp]`` without gathering them."""
    tp = tp_mesh.size()
    if vocab_size % tp:
        raise ValueError(f"Vocabulary size {vocab_size} is not divisible by TP size {tp}")
    vl = vocab_size // tp
    if local_logits.shape[-1] != vl:
        raise RuntimeError(f"Expected a vocabulary shard with last dimension {vl}, got {local_logits.shape[-1]}")
    v0 = tp_mesh.get_local_rank() * vl
    return _VocabParallelCE.apply(local_logits.reshape(-1, vl), labels.reshape(-1).to(local_logits.device),
                                  tp_mesh.get_group(), v0, reduction)


class _VocabParallelLMHeadCE(torch.autograd.Function):
    @staticmethod
    def forward(ctx, h, w, labels, group, v0, block_bytes, small):
        T, H = h.shape
        V = w.shape[0]
        labels = labels.reshape(-1).contiguous()
        # labels are in [0, vocab) or IGNORE (< 0): the kernels count labels >= 0
        inv = torch.empty(1, device=h.device, dtype=torch.float32)
        ext().ce_valid_inv(labels, inv)
        rows = max(128, min(T, int(block_bytes // (V * 2)) // 128 * 128))
        dh = torch.empty_like(h)
        dw = torch.empty(V, H, device=h.device, dtype=torch.float32)
        loss = torch.empty(1, device=h.device, dtype=torch.float32)
        for r0 in range(0, T, rows):
            r1 = min(T, r0 + rows)
            hb = h[r0:r1]
            lb = labels[r0:r1]
            logits = G.linear(hb, w)
            mx = torch.empty(r1 - r0, device=h.device)
            se = torch.empty(r1 - r0, device=h.device)
            ext().ce_row_stats(logits, mx, se)
            if small is not None:
                # one peer-memory kernel merges (max, sum-exp, target) of every rank
                local = lb - v0
                inside = (lb != IGNORE) & (local >= 0) & (local < V)
                tl = logits.gather(1, local.clamp(0, V - 1)[:, None])[:, 0].float()
                lse, tgt = small.lse_merge(mx, se, torch.where(inside, tl, torch.zeros_like(tl)))
                ext().ce_fwd_bwd(logits, lb, v0, inv, lse, True, None, True)
            else:
                gm = mx.clone()
                dist.all_reduce(gm, op=dist.ReduceOp.MAX, group=group)
                se = se * torch.exp(mx - gm)
                dist.all_reduce(se, op=dist.ReduceOp.SUM, group=group)
                lse = gm + torch.log(se)
                tgt = torch.empty(r1 - r0, device=h.device)
                ext().ce_fwd_bwd(logits, lb, v0, inv, lse, True, tgt, True)
                dist.all_reduce(tgt, op=dist.ReduceOp.SUM, group=group)
            # every rank holds the global (lse, target): the same fixed-order sum everywhere
            ext().ce_loss_reduce(lse.contiguous(), tgt.contiguous(), lb, inv, loss, r0 > 0)
            G.linear_dgrad(logits, w, out=dh[r0:r1])
            G.linear_wgrad(logits, hb, out=dw, accumulate=r0 > 0)
            del logits
        dwb = torch.empty(V, H, device=h.device, dtype=w.dtype)
        ext().cast_f32_to_bf16(dw, dwb)
        ctx.save_for_backward(dh, dwb)
        return loss.reshape(())

    @staticmethod
    def backward(ctx, g):
        dh, dw = ctx.saved_tensors
        return dh * g.to(dh.dtype), dw * g.to(dw.dtype), None, None, None, None, None


def vocab_parallel_lm_head_ce(h, w_local, labels, group, vocab_start: int, block_bytes: int = 4 << 30,
                              collectives: str = "auto"):
    """Mean CE of ``h @ w_local.T`` whose vocab is sharded over ``group`` (CUDA).

    ``h`` [T, H] (the gathered hidden states, identical on every TP rank);
    the returned gradient of ``h`` is this rank's partial, to be summed over
    the TP group by the caller's ``copy_to_tp`` boundary.  With NVLink peer
    access (``collectives`` not "nccl") the per-block statistics of all ranks
    are merged by one peer-memory kernel instead of three NCCL all-reduces."""
    small = None
    if collectives != "nccl":
        from ..comm.p2p import P2PSmallAllReduce

        small = P2PSmallAllReduce.get(group, h.device)
        if small is not None and h.reshape(-1, h.shape[-1]).shape[0] > small.cap:
            small = None
    return _VocabParallelLMHeadCE.apply(h.reshape(-1, h.shape[-1]).contiguous(), w_local, labels, group,
                                        vocab_start, block_bytes, small)
