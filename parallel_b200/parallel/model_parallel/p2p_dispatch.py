"""Expert-parallel token dispatch / combine over NVLink peer memory.

Same interface and semantics as ``TokenDispatcher`` (reference:
parallel/parallel/engine/model_parallel/token_dispatch.py:101-174), with the
data plane replaced by the peer-memory row kernels of ``csrc/comm.cu``:

* dispatch: every route's hidden row (and a 16-byte record: local expert id,
  score, source route) is stored by one warp straight into the owning rank's
  symmetric receive buffer, at the row given by the route counts of all
  ranks (one small all-gather of the per-destination counts; like the
  reference, the counts go to the host because they size the expert GEMMs);
  no staging sort / all-to-all / index_select.
* combine: the owner exposes its expert outputs in a symmetric buffer and
  each source rank pulls its tokens' top-k rows and sums them in fp32 in one
  kernel (the reference's all-to-all back + index_add).
* backward: dispatch's backward is a pull-and-sum (hidden) plus a pull (score
  gradients); combine's backward pushes each token's output gradient to its
  routes' rows at the owners.

Symmetric buffers rotate over two sets; one signal barrier per exchange
orders reuse (every rank finished exchange n-1 when a rank passes the
barrier of exchange n).
"""
from __future__ import annotations

import os

import torch
import torch.distributed as dist

from ...ops._ext import ext
from ...profiling import collective_profile
from ..comm.p2p import SymmBuffer, p2p_supported


class _Pool:
    """Two rotating sets of symmetric buffers: rows [cap, H] bf16 and 16-byte records [cap, 4] int32."""

    def __init__(self, group, device, cap: int, hidden: int):
        self.cap, self.hidden = cap, hidden
        self.rows = [SymmBuffer(cap * hidden, torch.bfloat16, device, group, "ep_rows") for _ in range(2)]
        self.recs = [SymmBuffer(cap * 4, torch.int32, device, group, "ep_records") for _ in range(2)]
        self.n = 0

    def next(self):
        k = self.n % 2
        self.n += 1
        return self.rows[k], self.recs[k]


class P2PTokenDispatcher:
    def __init__(self, partition, group, device):
        self.partition = partition
        self.group = group
        self.world_size = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        self.device = device
        self.limit_s = float(os.environ.get("PB_P2P_TIMEOUT_S", "60"))
        self.pool: _Pool | None = None

    @staticmethod
    def available(group, device) -> bool:
        return device.type == "cuda" and p2p_supported(group)

    def _ensure(self, routes: int, hidden: int) -> _Pool:
        cap = routes * self.world_size  # every route of every rank could target one owner
        if self.pool is None:
            self.pool = _Pool(self.group, self.device, cap, hidden)
        elif cap > self.pool.cap or hidden != self.pool.hidden:
            raise RuntimeError(f"P2P dispatch buffers were sized for {self.pool.cap} routes x {self.pool.hidden}; "
                               f"got {cap} x {hidden}")
        return self.pool

    def _barrier(self, buf: SymmBuffer) -> None:
        buf.barrier(0, self.limit_s)

    # ------------------------------------------------------------------ dispatch
    def dispatch(self, hidden_states, global_indices, scores):
        if global_indices.shape != scores.shape:
            raise ValueError("Expert indices and scores must have the same shape")
        tokens, top_k = global_indices.shape
        flat_e = global_indices.reshape(-1)
        dest = self.partition.owner(flat_e).to(torch.int64)
        order = torch.argsort(dest, stable=True)
        dest_sorted = dest[order]
        send = torch.bincount(dest, minlength=self.world_size).to(torch.int64)
        mat = torch.empty(self.world_size, self.world_size, dtype=torch.int64, device=send.device)
        with collective_profile("ep_all_gather", value=send, mode="split_counts", detail="route_counts"):
            dist.all_gather_into_tensor(mat.view(-1), send, group=self.group)
        m = mat.tolist()  # [src][dst]
        W, me = self.world_size, self.rank
        recv_total = sum(m[s][me] for s in range(W))
        offs_at_dst = torch.tensor([sum(m[s][d] for s in range(me)) for d in range(W)], device=send.device)
        starts = torch.tensor([sum(m[me][:d]) for d in range(W)], device=send.device)
        n = flat_e.numel()
        pos = torch.arange(n, device=send.device)
        dst_row_sorted = offs_at_dst[dest_sorted] + pos - starts[dest_sorted]
        # flat-route order (t*K + k): destination rank and row of every route
        dst_row = torch.empty_like(dst_row_sorted)
        dst_row[order] = dst_row_sorted
        src_of_recv = torch.repeat_interleave(torch.arange(W, device=send.device),
                                              torch.tensor([m[s][me] for s in range(W)], device=send.device))
        state = _P2PDispatchState(dest.to(torch.int32).contiguous(), dst_row.contiguous(), tokens, top_k,
                                  recv_total, src_of_recv)
        local_e = (flat_e - dest * self.partition.local_count).to(torch.int32)
        rh, rs = _DispatchFn.apply(hidden_states, scores, self, state, local_e, order)
        re = state.recv_experts
        return rh, re.unsqueeze(-1), rs.unsqueeze(-1), state

    def combine(self, expert_output: torch.Tensor, state):
        return _CombineFn.apply(expert_output, self, state)


class _P2PDispatchState:
    def __init__(self, route_rank, route_row, tokens, top_k, recv_total, src_of_recv):
        self.route_rank = route_rank  # int32 [T*K]: owner rank of each flat route
        self.route_row = route_row    # int64 [T*K]: row of the route in the owner's buffers
        self.num_source_tokens = tokens
        self.top_k = top_k
        self.recv_total = recv_total
        self.src_of_recv = src_of_recv  # [R] source rank of each received row
        self.recv_experts = None
        self.recv_src_route = None


class _DispatchFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, hidden, scores, disp, state, local_e, order):
        C = ext()
        T, H = hidden.shape
        K = state.top_k
        pool = disp._ensure(T * K, H)
        rows, recs = pool.next()
        n = T * K
        flat_route = torch.arange(n, device=hidden.device)
        rec = torch.zeros(n, 4, dtype=torch.int32, device=hidden.device)
        rec[:, 0] = local_e
        rec[:, 1] = scores.reshape(-1).to(torch.float32).view(torch.int32)
        rec[:, 2] = flat_route.to(torch.int32)
        h2 = hidden.reshape(T, H)
        h2 = h2 if h2.stride(-1) == 1 else h2.contiguous()
        tok = torch.div(flat_route, K, rounding_mode="floor")
        with collective_profile("ep_dispatch", value=hidden, mode="p2p", detail="routes"):
            C.row_scatter(h2, tok, state.route_rank, state.route_row, rows.peer_ptrs, H * 2)
            C.row_scatter(rec, flat_route, state.route_rank, state.route_row, recs.peer_ptrs, 16)
            disp._barrier(rows)
        R = state.recv_total
        rh = rows.tensor[: R * H].view(R, H).clone()
        rrec = recs.tensor[: R * 4].view(R, 4).clone()
        state.recv_experts = rrec[:, 0].to(torch.int64)
        state.recv_src_route = rrec[:, 2].to(torch.int64)
        rs = rrec[:, 1].contiguous().view(torch.float32).to(scores.dtype)
        ctx.disp, ctx.state, ctx.shape, ctx.sdtype = disp, state, (T, H), scores.dtype
        ctx.sshape = scores.shape
        return rh, rs

    @staticmethod
    def backward(ctx, g_h, g_s):
        C = ext()
        disp, state = ctx.disp, ctx.state
        T, H = ctx.shape
        K = state.top_k
        rows, recs = disp.pool.next()
        R = state.recv_total
        if g_h is None:
            g_h = torch.zeros(R, H, device=rows.tensor.device, dtype=torch.bfloat16)
        if g_s is None:
            g_s = torch.zeros(R, device=rows.tensor.device)
        rows.tensor[: R * H].view(R, H).copy_(g_h.reshape(R, H))
        rec = recs.tensor[: R * 4].view(R, 4)
        rec.zero_()
        rec[:, 0] = g_s.reshape(R).to(torch.float32).view(torch.int32)
        with collective_profile("ep_dispatch", value=g_h, mode="p2p_grad", detail="routes"):
            disp._barrier(rows)
            dh = torch.empty(T, H, device=g_h.device, dtype=torch.bfloat16)
            C.row_gather_sum(dh, state.route_rank, state.route_row, rows.peer_ptrs, H)
            gs = torch.empty(T * K, 4, dtype=torch.int32, device=g_h.device)
            C.row_gather(gs, state.route_rank, state.route_row, recs.peer_ptrs, 16)
        dscores = gs[:, 0].contiguous().view(torch.float32).view(ctx.sshape).to(ctx.sdtype)
        return dh, dscores, None, None, None, None


class _CombineFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, y, disp, state):
        C = ext()
        R, H = y.shape
        rows, _ = disp.pool.next()
        rows.tensor[: R * H].view(R, H).copy_(y)
        T = state.num_source_tokens
        out = torch.empty(T, H, device=y.device, dtype=torch.bfloat16)
        with collective_profile("ep_combine", value=y, mode="p2p", detail="routes"):
            disp._barrier(rows)
            C.row_gather_sum(out, state.route_rank, state.route_row, rows.peer_ptrs, H)
        ctx.disp, ctx.state, ctx.R, ctx.ydtype = disp, state, R, y.dtype
        return out

    @staticmethod
    def backward(ctx, g):
        C = ext()
        disp, state = ctx.disp, ctx.state
        K = state.top_k
        T, H = g.shape
        rows, _ = disp.pool.next()
        g2 = g if g.stride(-1) == 1 else g.contiguous()
        flat_route = torch.arange(T * K, device=g.device)
        tok = torch.div(flat_route, K, rounding_mode="floor")
        with collective_profile("ep_combine", value=g, mode="p2p_grad", detail="routes"):
            C.row_scatter(g2.to(torch.bfloat16), tok, state.route_rank, state.route_row, rows.peer_ptrs, H * 2)
            disp._barrier(rows)
        gy = rows.tensor[: ctx.R * H].view(ctx.R, H).clone().to(ctx.ydtype)
        return gy, None, None
