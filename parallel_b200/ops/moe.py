"""Mixture-of-experts pieces: top-k router, expert SwiGLU MLPs, Switch aux loss.

Semantics follow HF Qwen3-MoE, which the reference trains unchanged:
* router (transformers/models/qwen3_moe/modeling_qwen3_moe.py,
  Qwen3MoeTopKRouter): logits = x W^T, fp32 softmax, top-k, optional
  renormalisation; the *softmax probabilities* are what the model records
  as "router_logits";
* experts (Qwen3MoeExperts): gate_up_proj[e] is [2I, H] with the gate half
  first; y = sum_k w_k * down(silu(g) * u);
* aux loss (load_balancing_loss_func): softmax is applied AGAIN to the
  recorded probabilities (the double softmax the reference inherits, also
  copied by parallel/parallel/engine/model_parallel/sequence_parallel.py:250).

Routes whose expert index equals ``num_local`` (the "sentinel" the
replicated-token expert parallelism uses for experts owned by other ranks,
parallel/parallel/engine/model_parallel/expert_parallel.py:50-60) are
skipped explicitly.

On CUDA the expert MLPs run the tcgen05 SwiGLU GEMM per expert on rows
sorted by expert; on CPU the plain PyTorch loop runs.
"""
from __future__ import annotations

import torch
import torch.nn.functional as F

from . import gemm as G
from ._ext import ext


def route(x2: torch.Tensor, w: torch.Tensor, top_k: int, norm_topk_prob: bool):
    """Returns (probs [T, E] fp32 softmax, top-k weights [T, k], top-k index [T, k])."""
    from .functional import linear as _linear

    logits = _linear(x2.contiguous(), w) if (x2.is_cuda and _gemm_ok(x2, w)) else F.linear(x2, w)
    probs = torch.softmax(logits, dim=-1, dtype=torch.float32)
    top_v, top_i = torch.topk(probs, top_k, dim=-1)
    if norm_topk_prob:
        top_v = top_v / top_v.sum(dim=-1, keepdim=True)
    return probs, top_v.to(probs.dtype), top_i


def _gemm_ok(x2, w) -> bool:
    return (x2.dtype == torch.bfloat16 and w.dtype == torch.bfloat16 and x2.shape[-1] % 8 == 0
            and w.is_contiguous() and x2.shape[0] > 0)


class _ExpertsFn(torch.autograd.Function):
    """Expert SwiGLU MLPs over expert-sorted rows.

    xs: [N, H] rows sorted by expert; counts: python list of rows per expert;
    scores: [N] routing weights (fp32); w_gu [E, 2I, H]; w_d [E, H, I].
    Returns ys [N, H] = score * down(silu(g) * u).
    """

    @staticmethod
    def forward(ctx, xs, scores, w_gu, w_d, counts):
        N, H = xs.shape
        I = w_d.shape[2]
        ys = torch.empty_like(xs)
        y_raw = torch.empty_like(xs)
        gu_all = torch.empty(N, 2 * I, device=xs.device, dtype=xs.dtype)
        h_all = torch.empty(N, I, device=xs.device, dtype=xs.dtype)
        r = 0
        for e, n in enumerate(counts):
            if n == 0:
                continue
            xe = xs[r:r + n]
            ext().gemm(xe, w_gu[e], h_all[r:r + n], False, False, G.EPI_SWIGLU, 1.0, gu_all[r:r + n], I, I)
            ext().gemm(h_all[r:r + n], w_d[e], y_raw[r:r + n], False, False, G.EPI_STORE_BF16, 1.0)
            r += n
        ys.copy_(y_raw * scores[:, None].to(y_raw.dtype))
        ctx.save_for_backward(xs, scores, w_gu, w_d, gu_all, h_all, y_raw)
        ctx.counts = counts
        return ys

    @staticmethod
    def backward(ctx, dys):
        xs, scores, w_gu, w_d, gu_all, h_all, y_raw = ctx.saved_tensors
        counts = ctx.counts
        I = w_d.shape[2]
        dys = dys.contiguous()
        dscores = (dys.float() * y_raw.float()).sum(-1)
        dy_s = (dys * scores[:, None].to(dys.dtype)).contiguous()
        dxs = torch.zeros_like(xs)
        dw_gu = torch.zeros_like(w_gu)
        dw_d = torch.zeros_like(w_d)
        dh = torch.empty(xs.shape[0], I, device=xs.device, dtype=xs.dtype)
        dgu = torch.empty_like(gu_all)
        r = 0
        for e, n in enumerate(counts):
            if n == 0:
                continue
            sl = slice(r, r + n)
            G.linear_dgrad(dy_s[sl], w_d[e], out=dh[sl])
            G.linear_wgrad(dy_s[sl], h_all[sl], out=dw_d[e])
            ext().swiglu_bwd(dh[sl], gu_all[sl], dgu[sl])
            G.linear_dgrad(dgu[sl], w_gu[e], out=dxs[sl])
            G.linear_wgrad(dgu[sl], xs[sl], out=dw_gu[e])
            r += n
        return dxs, dscores.to(scores.dtype), dw_gu, dw_d, None


def experts_forward(x2: torch.Tensor, top_k_index: torch.Tensor, top_k_weights: torch.Tensor,
                    w_gu: torch.Tensor, w_d: torch.Tensor) -> torch.Tensor:
    """sum_k w_k * expert_{idx_k}(x) for routes with idx < num_local."""
    E = w_gu.shape[0]
    T, K = top_k_index.shape
    if not x2.is_cuda:
        out = torch.zeros_like(x2)
        for e in range(E):
            tok, kpos = torch.where(top_k_index == e)
            if tok.numel() == 0:
                continue
            g, u = F.linear(x2[tok], w_gu[e]).chunk(2, dim=-1)
            y = F.linear(F.silu(g) * u, w_d[e]) * top_k_weights[tok, kpos, None]
            out = out.index_add(0, tok, y.to(out.dtype))
        return out
    flat_e = top_k_index.reshape(-1)
    valid = flat_e < E
    order = torch.argsort(torch.where(valid, flat_e, E), stable=True)
    counts_t = torch.bincount(flat_e[valid], minlength=E)
    counts = counts_t.tolist()
    n_valid = int(sum(counts))
    order = order[:n_valid]
    tok = order // K
    xs = x2.index_select(0, tok).contiguous()
    scores = top_k_weights.reshape(-1).index_select(0, order)
    ys = _ExpertsFn.apply(xs, scores, w_gu, w_d, counts)
    out = torch.zeros_like(x2)
    return out.index_add(0, tok, ys)


def load_balancing_loss(router_probs: tuple, num_experts: int, top_k: int) -> torch.Tensor:
    """HF load_balancing_loss_func (no attention mask), double softmax included."""
    cat = torch.cat([p.to(router_probs[0].device) for p in router_probs], dim=0)
    routing_weights = torch.softmax(cat, dim=-1)
    _, selected = torch.topk(routing_weights, top_k, dim=-1)
    expert_mask = F.one_hot(selected, num_experts)
    tokens_per_expert = torch.mean(expert_mask.float(), dim=0)
    router_prob_per_expert = torch.mean(routing_weights, dim=0)
    return torch.sum(tokens_per_expert * router_prob_per_expert.unsqueeze(0)) * num_experts
