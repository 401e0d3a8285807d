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

On CUDA the router's softmax / top-k / renormalisation / histogram and the
loss statistics are fused kernels (csrc/router.cu) and the expert MLPs run as
grouped tcgen05 GEMMs (csrc/gemm_grouped.cu, one launch per product for all
experts); on CPU the plain PyTorch code runs.
"""
from __future__ import annotations

import torch
import torch.nn.functional as F

from . import gemm as G
from ._ext import ext


class _RouterFn(torch.autograd.Function):
    """Softmax + top-k + renormalisation (+ route histogram) of bf16 router
    logits in one kernel (csrc/router.cu); the backward folds the gradients of
    the probabilities (auxiliary loss) and of the selected weights."""

    @staticmethod
    def forward(ctx, logits, top_k, renorm, counts):
        T, E = logits.shape
        probs = torch.empty(T, E, device=logits.device, dtype=torch.float32)
        topv = torch.empty(T, top_k, device=logits.device, dtype=torch.float32)
        topi = torch.empty(T, top_k, device=logits.device, dtype=torch.int64)
        ext().router_fwd(logits, top_k, renorm, probs, topv, topi, counts)
        ctx.save_for_backward(probs, topi)
        ctx.renorm = renorm
        ctx.mark_non_differentiable(topi)
        return probs, topv, topi

    @staticmethod
    def backward(ctx, dprobs, dtopv, _):
        probs, topi = ctx.saved_tensors
        T, E = probs.shape
        if dtopv is None:
            dtopv = torch.zeros_like(topi, dtype=torch.float32)
        dtopv = dtopv.float().contiguous()
        if dprobs is not None:
            dprobs = dprobs.float().contiguous()
        dl = torch.empty(T, E, device=probs.device, dtype=torch.bfloat16)
        ext().router_bwd(probs, dprobs, dtopv, topi, ctx.renorm, dl)
        return dl, None, None, None


def _router_kernel_ok(logits: torch.Tensor, top_k: int) -> bool:
    return (logits.is_cuda and logits.dtype == torch.bfloat16 and logits.dim() == 2 and logits.stride(1) == 1
            and 1 <= logits.shape[1] <= 256 and 1 <= top_k <= min(16, logits.shape[1]))


def route(x2: torch.Tensor, w: torch.Tensor, top_k: int, norm_topk_prob: bool, counts: torch.Tensor | None = None):
    """Returns (probs [T, E] fp32 softmax, top-k weights [T, k], top-k index [T, k]).
    On CUDA ``counts`` (int32 [E]), when given, accumulates the route histogram."""
    from .functional import linear as _linear

    logits = _linear(x2.contiguous(), w) if (x2.is_cuda and _gemm_ok(x2, w)) else F.linear(x2, w)
    if _router_kernel_ok(logits, top_k):
        return _RouterFn.apply(logits, top_k, bool(norm_topk_prob), counts)
    probs = torch.softmax(logits, dim=-1, dtype=torch.float32)
    top_v, top_i = torch.topk(probs, top_k, dim=-1)
    if norm_topk_prob:
        top_v = top_v / top_v.sum(dim=-1, keepdim=True)
    return probs, top_v.to(probs.dtype), top_i


def _gemm_ok(x2, w) -> bool:
    return (x2.dtype == torch.bfloat16 and w.dtype == torch.bfloat16 and x2.shape[-1] % 8 == 0
            and w.is_contiguous() and x2.shape[0] > 0)


def _padded_layout(counts: list, device):
    """Rows of expert e at a 128-aligned offset: (offsets list, padded total, index of each sorted row)."""
    offs, o = [], 0
    for n in counts:
        offs.append(o)
        o += -(-n // 128) * 128
    pos = torch.cat([torch.arange(n, device=device) + off for n, off in zip(counts, offs) if n > 0]) \
        if any(counts) else torch.zeros(0, dtype=torch.int64, device=device)
    return offs, max(o, 128), pos


def _rows_work(counts, offs, n_tiles: int, device) -> torch.Tensor:
    """Grouped-GEMM rows-mode work table {expert, M tile, N tile, 0}."""
    items = [(e, off // 128 + t, tn, 0) for e, (n, off) in enumerate(zip(counts, offs)) if n > 0
             for t in range(-(-n // 128)) for tn in range(n_tiles)]
    return torch.tensor(items or [(0, 0, 0, 0)], dtype=torch.int32, device=device)[: len(items)]


def _k_work(counts, m_group: int, n: int, device):
    """Grouped-GEMM k-mode work table and per-expert row ranges (64-row multiples)."""
    items = [(e, tm, tn, 0) for e, c in enumerate(counts) if c > 0
             for tm in range(-(-m_group // 128)) for tn in range(-(-n // 128))]
    return torch.tensor(items or [(0, 0, 0, 0)], dtype=torch.int32, device=device)[: len(items)]


class _ExpertsFn(torch.autograd.Function):
    """Expert SwiGLU MLPs over expert-sorted rows, as grouped tcgen05 GEMMs.

    xs: [N, H] rows sorted by expert; counts: python list of rows per expert;
    scores: [N] routing weights (fp32); w_gu [E, 2I, H]; w_d [E, H, I].
    Returns ys [N, H] = score * down(silu(g) * u).  Rows are laid out per
    expert at 128-row aligned offsets with zero rows in between (one launch
    per product: gate/up + SwiGLU, down; backward: down input-grad, down
    weight-grad, SwiGLU backward, gate/up input-grad, gate/up weight-grad).
    """

    @staticmethod
    def forward(ctx, xs, scores, w_gu, w_d, counts):
        N, H = xs.shape
        E, I = w_d.shape[0], w_d.shape[2]
        offs, n_pad, pos = _padded_layout(counts, xs.device)
        x_pad = torch.zeros(n_pad, H, device=xs.device, dtype=xs.dtype)
        x_pad[pos] = xs
        gu_pad = torch.empty(n_pad, 2 * I, device=xs.device, dtype=xs.dtype)
        h_pad = torch.empty(n_pad, I, device=xs.device, dtype=xs.dtype)
        w_gu = w_gu.contiguous()
        w_d = w_d.contiguous()
        C = ext()
        C.gemm_grouped(1, x_pad, w_gu, h_pad, _rows_work(counts, offs, -(-I // 128), xs.device), None, False,
                       G.EPI_SWIGLU, 1.0, gu_pad, I, I)
        y_pad = torch.empty(n_pad, H, device=xs.device, dtype=xs.dtype)
        C.gemm_grouped(1, h_pad, w_d, y_pad, _rows_work(counts, offs, -(-H // 128), xs.device), None, False,
                       G.EPI_STORE_BF16, 1.0)
        y_raw = y_pad[pos]
        ys = y_raw * scores[:, None].to(y_raw.dtype)
        ctx.save_for_backward(x_pad, scores, w_gu, w_d, gu_pad, h_pad, y_raw, pos)
        ctx.counts, ctx.offs = counts, offs
        return ys

    @staticmethod
    def backward(ctx, dys):
        x_pad, scores, w_gu, w_d, gu_pad, h_pad, y_raw, pos = ctx.saved_tensors
        counts, offs = ctx.counts, ctx.offs
        E, H, I = w_d.shape
        n_pad = x_pad.shape[0]
        dev = x_pad.device
        dys = dys.contiguous()
        dscores = (dys.float() * y_raw.float()).sum(-1)
        dy_pad = torch.zeros(n_pad, H, device=dev, dtype=dys.dtype)
        dy_pad[pos] = dys * scores[:, None].to(dys.dtype)
        krange = torch.tensor([[off, off + -(-n // 64) * 64] for n, off in zip(counts, offs)], dtype=torch.int32,
                              device=dev)
        C = ext()
        # down projection: dh = dy W_d (rows), dW_d[e] = dy_e^T h_e (k)
        dh_pad = torch.empty(n_pad, I, device=dev, dtype=dys.dtype)
        C.gemm_grouped(1, dy_pad, w_d, dh_pad, _rows_work(counts, offs, -(-I // 128), dev), None, True,
                       G.EPI_STORE_BF16, 1.0)
        dw_d = torch.zeros_like(w_d)
        C.gemm_grouped(2, dy_pad, h_pad, dw_d, _k_work(counts, H, I, dev), krange, True, G.EPI_STORE_BF16, 1.0)
        dgu = torch.empty_like(gu_pad)
        C.swiglu_bwd(dh_pad, gu_pad, dgu)
        # gate/up projection: dx = dgu W_gu (rows), dW_gu[e] = dgu_e^T x_e (k)
        dx_pad = torch.empty(n_pad, H, device=dev, dtype=dys.dtype)
        C.gemm_grouped(1, dgu, w_gu, dx_pad, _rows_work(counts, offs, -(-H // 128), dev), None, True,
                       G.EPI_STORE_BF16, 1.0)
        dw_gu = torch.zeros_like(w_gu)
        C.gemm_grouped(2, dgu, x_pad, dw_gu, _k_work(counts, 2 * I, H, dev), krange, True, G.EPI_STORE_BF16, 1.0)
        return dx_pad[pos], dscores.to(scores.dtype), dw_gu, dw_d, None


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


class _AuxStatsFn(torch.autograd.Function):
    """Per-expert statistics of the load-balancing loss over recorded router
    probabilities p [R, E]: (top-k selection counts of s = softmax(p), sums of s
    over the rows); differentiable in the sums (csrc/router.cu)."""

    @staticmethod
    def forward(ctx, probs, top_k):
        E = probs.shape[1]
        counts = torch.zeros(E, device=probs.device, dtype=torch.float32)
        ssum = torch.zeros(E, device=probs.device, dtype=torch.float32)
        ext().aux_stats(probs, top_k, counts, ssum)
        ctx.save_for_backward(probs)
        ctx.mark_non_differentiable(counts)
        return counts, ssum

    @staticmethod
    def backward(ctx, _, gsum):
        (probs,) = ctx.saved_tensors
        dp = torch.empty_like(probs)
        ext().aux_stats_bwd(probs, gsum.float().contiguous(), dp)
        return dp, None


def aux_loss_stats(probs: torch.Tensor, top_k: int):
    """(counts [E], sums [E]) of the double-softmax load-balancing loss; the
    counts sum the top-k selections of softmax(probs) over rows and slots."""
    E = probs.shape[-1]
    if probs.is_cuda and probs.dtype == torch.float32 and probs.dim() == 2 and 1 <= E <= 256 \
            and 1 <= top_k <= min(16, E):
        return _AuxStatsFn.apply(probs.contiguous(), top_k)
    s = torch.softmax(probs, dim=-1)
    selected = torch.topk(s, top_k, dim=-1).indices
    counts = F.one_hot(selected, probs.shape[1]).float().sum(dim=(0, 1))
    return counts, s.sum(dim=0)


def load_balancing_loss(router_probs: tuple, num_experts: int, top_k: int) -> torch.Tensor:
    """HF load_balancing_loss_func (no attention mask), double softmax included."""
    cat = torch.cat([p.to(router_probs[0].device) for p in router_probs], dim=0)
    if cat.is_cuda:
        counts, ssum = aux_loss_stats(cat.float(), top_k)
        R = cat.shape[0]
        return torch.sum((counts / R) * (ssum / R)) * num_experts
    routing_weights = torch.softmax(cat, dim=-1)
    _, selected = torch.topk(routing_weights, top_k, dim=-1)
    expert_mask = F.one_hot(selected, num_experts)
    tokens_per_expert = torch.mean(expert_mask.float(), dim=0)
    router_prob_per_expert = torch.mean(routing_weights, dim=0)
    return torch.sum(tokens_per_expert * router_prob_per_expert.unsqueeze(0)) * num_experts
