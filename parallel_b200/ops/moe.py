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

On CUDA the router's softmax / top-k / renormalisation and the loss
statistics are fused kernels (csrc/router.cu).  The experts run on a
device-resident routing plan (csrc/moe.cu): a stable counting sort on the GPU
places every route in a 128-row padded expert-major matrix, the expert MLPs
are grouped tcgen05 GEMMs over that matrix whose tile count is read on the
device (csrc/gemm_grouped.cu), and the combine sums each token's routes with
their routing weights in fp32.  No count reaches the host, so MoE layers run
without a synchronisation and can be captured in a CUDA graph.  A transport
object says where the routed rows go: this device (``LocalExpertTransport``;
with ``local_only`` the replicated-token expert parallelism keeps just the
routes to this rank's experts, the reference's sentinel routes of
parallel/parallel/engine/model_parallel/expert_parallel.py:50-60) or the EP
group's peer memory (``PeerExpertTransport``).  On CPU the plain PyTorch
code runs, where routes with an expert index >= the local expert count are
skipped.
"""
from __future__ import annotations

from dataclasses import dataclass

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


def route(x2: torch.Tensor, w: torch.Tensor, top_k: int, norm_topk_prob: bool, counts: torch.Tensor | None = None,
          logit_bias: torch.Tensor | None = None):
    """Returns (probs [T, E] fp32 softmax, top-k weights [T, k], top-k index [T, k]).
    On CUDA ``counts`` (int32 [E]), when given, accumulates the route histogram.
    ``logit_bias`` ([E], optional) is added to the logits (a benchmark knob
    that skews the routing; Qwen3-MoE routers have no bias)."""
    from .functional import linear as _linear

    logits = _linear(x2.contiguous(), w) if (x2.is_cuda and _gemm_ok(x2, w)) else F.linear(x2, w)
    if logit_bias is not None:
        logits = logits + logit_bias.to(logits.dtype)
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


# --------------------------------------------------------------------------- device-resident routing
@dataclass
class RoutePlan:
    """Device tensors describing one MoE layer's routing (``csrc/moe.cu``)."""

    route_owner: torch.Tensor  # int32 [T*K]: owner index of each route (-1: not kept)
    route_row: torch.Tensor    # int32 [T*K]: row of the route in the owner's padded matrix
    own_cnt: torch.Tensor      # int32 [E_loc]: rows routed to each local expert
    own_off: torch.Tensor      # int32 [E_loc]: first padded row of each local expert
    krange: torch.Tensor       # int32 [E_loc, 2]: weight-gradient row range of each local expert
    tile_expert: torch.Tensor  # int32 [tiles_cap]: local expert of each 128-row tile
    n_tiles: torch.Tensor      # int32 [1]: live tiles of the padded matrix
    top_k: int

    @property
    def rows_cap(self) -> int:
        return 128 * self.tile_expert.numel()


def tiles_capacity(routes_in: int, num_local: int) -> int:
    """Worst-case 128-row tiles of an owner's padded matrix when at most
    ``routes_in`` routes reach it: every expert rounds up by < 128 rows and an
    expert without routes still takes one tile."""
    return -(-(routes_in + 128 * num_local) // 128)


def plan_routes(topi: torch.Tensor, hist: torch.Tensor, my_row: int, num_local: int, ep_rank: int,
                local_only: bool, tiles_cap: int) -> RoutePlan:
    n = topi.numel()
    dev = topi.device
    i32 = dict(dtype=torch.int32, device=dev)
    plan = RoutePlan(torch.empty(n, **i32), torch.empty(n, **i32), torch.empty(num_local, **i32),
                     torch.empty(num_local, **i32), torch.empty(num_local, 2, **i32), torch.empty(tiles_cap, **i32),
                     torch.empty(1, **i32), topi.shape[-1])
    ext().moe_plan(topi.contiguous(), hist, my_row, num_local, ep_rank, local_only, plan.route_owner, plan.route_row,
                   plan.own_cnt, plan.own_off, plan.krange, plan.tile_expert, plan.n_tiles)
    return plan


class LocalExpertTransport:
    """Routes whose experts live on this device: the padded expert matrix, the
    expert outputs and the gradients are ordinary device tensors.

    ``local_only`` keeps only the routes to this rank's experts (the
    replicated-token expert parallelism, where every rank routes every token
    and ``ep_rank`` owns experts [ep_rank * num_local, (ep_rank + 1) * num_local))."""

    def __init__(self, num_local: int, num_experts: int | None = None, ep_rank: int = 0, local_only: bool = False):
        self.num_local, self.ep_rank, self.local_only = num_local, ep_rank, local_only
        self.num_experts = num_local if num_experts is None else num_experts

    def _histogram(self, topi: torch.Tensor, num_experts: int):
        hist = torch.empty(1, num_experts, dtype=torch.float32, device=topi.device)
        ext().moe_hist(topi, hist, 0)
        return hist, 0

    def routes_in(self, routes: int) -> int:
        return routes

    def plan(self, topi: torch.Tensor, num_experts: int) -> RoutePlan:
        topi = topi.contiguous()
        hist, row = self._histogram(topi, num_experts)
        cap = tiles_capacity(self.routes_in(topi.numel()), self.num_local)
        return plan_routes(topi, hist, row, self.num_local, self.ep_rank, self.local_only, cap)

    def _pad(self, src_ptr: int, ld: int, dst: torch.Tensor, plan: RoutePlan) -> None:
        ext().moe_copy_pad(src_ptr, ld, dst, plan.tile_expert, plan.n_tiles, plan.own_cnt, plan.own_off)

    def dispatch(self, x2: torch.Tensor, plan: RoutePlan) -> torch.Tensor:
        """Padded expert matrix [rows_cap, H] of the routed rows (zero padding)."""
        H = x2.shape[1]
        x_pad = torch.empty(plan.rows_cap, H, device=x2.device, dtype=x2.dtype)
        ext().moe_dispatch(x2, plan.top_k, plan.route_owner, plan.route_row, [x_pad.data_ptr()], H)
        self._pad(x_pad.data_ptr(), H, x_pad, plan)
        return x_pad

    def output_buffer(self, plan: RoutePlan, H: int, like: torch.Tensor):
        buf = torch.empty(plan.rows_cap, H, device=like.device, dtype=like.dtype)
        return buf, [buf.data_ptr()]

    def combine(self, handle, plan: RoutePlan, weights: torch.Tensor, out: torch.Tensor, keep) -> None:
        ext().moe_combine(out, keep, weights, plan.route_owner, plan.route_row, handle, out.shape[1])

    def combine_backward(self, dout: torch.Tensor, keep: torch.Tensor, weights: torch.Tensor, plan: RoutePlan):
        H = dout.shape[1]
        dy_pad = torch.empty(plan.rows_cap, H, device=dout.device, dtype=dout.dtype)
        dw = torch.empty(weights.shape, device=dout.device, dtype=torch.float32)
        ext().moe_combine_bwd(dout, keep, weights, plan.route_owner, plan.route_row, [dy_pad.data_ptr()], H, dw)
        self._pad(dy_pad.data_ptr(), H, dy_pad, plan)
        return dy_pad, dw

    def grad_buffer(self, plan: RoutePlan, H: int, like: torch.Tensor):
        return self.output_buffer(plan, H, like)

    def gather_grad(self, handle, plan: RoutePlan, dx: torch.Tensor) -> None:
        ext().moe_combine(dx, None, None, plan.route_owner, plan.route_row, handle, dx.shape[1])


_NO_WORK: dict = {}
_K_WORK: dict = {}


def _empty_work(device) -> torch.Tensor:
    key = str(device)
    if key not in _NO_WORK:
        _NO_WORK[key] = torch.zeros(0, 4, dtype=torch.int32, device=device)
    return _NO_WORK[key]


def _k_work(num_local: int, m_group: int, n: int, device) -> torch.Tensor:
    """Weight-gradient work items {expert, M tile, N tile, 0} of every local
    expert (each expert's K range comes from the route plan); N tiles are as
    wide as the kernel's k-mode tile for this N."""
    bn = int(ext().grouped_tile_n(2, n))
    key = (num_local, m_group, n, bn, str(device))
    if key not in _K_WORK:
        items = [(e, tm, tn, 0) for e in range(num_local) for tm in range(-(-m_group // 128))
                 for tn in range(-(-n // bn))]
        _K_WORK[key] = torch.tensor(items, dtype=torch.int32, device=device)
    return _K_WORK[key]


class _RoutedExpertsFn(torch.autograd.Function):
    """Dispatch -> expert SwiGLU MLPs -> router-weighted combine, as one
    autograd node with every size on the device.

    x2 [T, H] bf16, weights [T, K] fp32 routing weights, topi [T, K] global
    expert ids, w_gu [E_loc, 2I, H], w_d [E_loc, H, I].  Forward: the routing
    plan, the rows into the owners' padded expert matrices, the gate/up
    grouped GEMM with the SwiGLU epilogue, the down grouped GEMM, then
    out[t] = sum_k w[t,k] * y[route] (fp32 sums).  Backward: dw[t,k] =
    <dout[t], y[route]>, w * dout into the owners' matrices, the down input /
    weight gradients, SwiGLU backward, the gate/up input / weight gradients,
    and each token's input gradient summed over its routes."""

    @staticmethod
    def forward(ctx, x2, weights, topi, w_gu, w_d, transport):
        C = ext()
        T, H = x2.shape
        E_loc, _, I = w_d.shape
        plan = transport.plan(topi, transport.num_experts)
        x_pad = transport.dispatch(x2.contiguous(), plan)
        rows = plan.rows_cap
        gu_pad = torch.empty(rows, 2 * I, device=x2.device, dtype=x2.dtype)
        h_pad = torch.empty(rows, I, device=x2.device, dtype=x2.dtype)
        w_gu, w_d = w_gu.contiguous(), w_d.contiguous()
        none = _empty_work(x2.device)
        C.gemm_grouped(1, x_pad, w_gu, h_pad, none, None, False, G.EPI_SWIGLU, 1.0, gu_pad, I, I,
                       tile_expert=plan.tile_expert, n_tiles=plan.n_tiles)
        y_buf, handle = transport.output_buffer(plan, H, x2)
        C.gemm_grouped(1, h_pad, w_d, y_buf, none, None, False, G.EPI_STORE_BF16, 1.0,
                       tile_expert=plan.tile_expert, n_tiles=plan.n_tiles)
        w32 = weights.detach().float().contiguous()
        keep = torch.empty(T * plan.top_k, H, device=x2.device, dtype=x2.dtype)
        out = torch.empty(T, H, device=x2.device, dtype=x2.dtype)
        transport.combine(handle, plan, w32, out, keep)
        ctx.save_for_backward(x_pad, gu_pad, h_pad, keep, w32, w_gu, w_d)
        ctx.plan, ctx.transport, ctx.wdtype = plan, transport, weights.dtype
        return out

    @staticmethod
    def backward(ctx, dout):
        C = ext()
        x_pad, gu_pad, h_pad, keep, w32, w_gu, w_d = ctx.saved_tensors
        plan, transport = ctx.plan, ctx.transport
        E_loc, H, I = w_d.shape
        dev = dout.device
        none = _empty_work(dev)
        dy_pad, dw = transport.combine_backward(dout.contiguous().to(keep.dtype), keep, w32, plan)
        # down projection: dh = dy W_d (rows), dW_d[e] = dy_e^T h_e (k)
        dh_pad = torch.empty(plan.rows_cap, I, device=dev, dtype=keep.dtype)
        C.gemm_grouped(1, dy_pad, w_d, dh_pad, none, None, True, G.EPI_STORE_BF16, 1.0,
                       tile_expert=plan.tile_expert, n_tiles=plan.n_tiles)
        dw_d = torch.empty_like(w_d)
        C.gemm_grouped(2, dy_pad, h_pad, dw_d, _k_work(E_loc, H, I, dev), plan.krange, True, G.EPI_STORE_BF16, 1.0)
        dgu = torch.empty_like(gu_pad)
        C.swiglu_bwd(dh_pad, gu_pad, dgu, plan.n_tiles)
        # gate/up projection: dx = dgu W_gu (rows, into the exchange buffer), dW_gu[e] = dgu_e^T x_e (k)
        dx_buf, handle = transport.grad_buffer(plan, H, keep)
        C.gemm_grouped(1, dgu, w_gu, dx_buf, none, None, True, G.EPI_STORE_BF16, 1.0,
                       tile_expert=plan.tile_expert, n_tiles=plan.n_tiles)
        dw_gu = torch.empty_like(w_gu)
        C.gemm_grouped(2, dgu, x_pad, dw_gu, _k_work(E_loc, 2 * I, H, dev), plan.krange, True, G.EPI_STORE_BF16,
                       1.0)
        dx = torch.empty(dout.shape[0], H, device=dev, dtype=keep.dtype)
        transport.gather_grad(handle, plan, dx)
        return dx, dw.to(ctx.wdtype), None, dw_gu, dw_d, None


def routed_experts_supported(x2: torch.Tensor, w_gu: torch.Tensor, num_experts: int) -> bool:
    return (x2.is_cuda and x2.dtype == torch.bfloat16 and w_gu.dtype == torch.bfloat16 and x2.shape[-1] % 8 == 0
            and w_gu.shape[1] % 16 == 0 and 1 <= num_experts <= 256)


def routed_experts(x2, weights, topi, w_gu, w_d, transport):
    """sum_k w_k * expert_{idx_k}(x) on the device path (see ``_RoutedExpertsFn``)."""
    return _RoutedExpertsFn.apply(x2, weights, topi, w_gu, w_d, transport)


def experts_forward(x2: torch.Tensor, top_k_index: torch.Tensor, top_k_weights: torch.Tensor,
                    w_gu: torch.Tensor, w_d: torch.Tensor) -> torch.Tensor:
    """sum_k w_k * expert_{idx_k}(x) for routes with idx < num_local (this
    device owns every expert it is given)."""
    E = w_gu.shape[0]
    if x2.is_cuda and routed_experts_supported(x2, w_gu, E):
        return routed_experts(x2, top_k_weights, top_k_index, w_gu, w_d, LocalExpertTransport(E))
    out = torch.zeros_like(x2)
    for e in range(E):
        tok, kpos = torch.where(top_k_index == e)
        if tok.numel() == 0:
            continue
        g, u = F.linear(x2[tok], w_gu[e]).chunk(2, dim=-1)
        y = F.linear(F.silu(g) * u, w_d[e]) * top_k_weights[tok, kpos, None]
        out = out.index_add(0, tok, y.to(out.dtype))
    return out


class _AuxStatsFn(torch.autograd.Function):
    """Per-expert statistics of the load-balancing loss over recorded router
    probabilities p [R, E]: (top-k selection counts of s = softmax(p), sums of s
    over the rows); differentiable in the sums (csrc/router.cu)."""

    @staticmethod
    def forward(ctx, probs, top_k):
        E = probs.shape[1]
        counts = torch.empty(E, device=probs.device, dtype=torch.float32)
        ssum = torch.empty(E, device=probs.device, dtype=torch.float32)
        ext().aux_stats(probs, top_k, counts, ssum)  # overwritten, summed in a fixed order
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
