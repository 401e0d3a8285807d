"""Expert-parallel token exchange over NVLink peer memory, without host syncs.

``PeerExpertTransport`` plugs into ``ops.moe.routed_experts`` (one autograd
node for dispatch -> expert GEMMs -> combine) for the sequence-parallel
expert parallelism: each rank routes its own tokens and the owners of the
chosen experts compute them.  Everything the exchange needs is sized on the
device:

* plan: each rank's route histogram over the global experts is written as
  its row of a [W, E] matrix and summed over the EP group (NVLink small
  all-reduce, or NCCL), which gives every rank every histogram; the plan
  kernel then derives every owner's padded expert layout and the destination
  (owner, row) of each of this rank's routes (``csrc/moe.cu``);
* dispatch: one kernel stores each route's hidden row straight into its
  owner's receive matrix (the permutation happens in the store); after a
  signal barrier the owner copies the live rows out into its padded expert
  matrix and zeroes the padding;
* the down-projection GEMM writes the expert outputs into this rank's
  exchange buffer; after a barrier each source rank pulls its routes' rows
  and sums them with the routing weights (fp32) - the combine;
* backward mirrors it: the routing-weight gradient and the weighted output
  gradient per route, pushed to the owners; the input-gradient GEMM writes
  into the exchange buffer and each source rank pulls and sums its routes.

Buffers are worst-case sized from the host-known token count (every route of
every rank could pick this owner), so no count ever reaches the host and an
MoE step can be captured in a CUDA graph.  Two rotating buffer sets with one
barrier per exchange order reuse: a rank writes a set only after the barrier
of the exchange in between, which every rank reaches after its reads of the
set's previous use.

Reference counterpart: ``parallel/parallel/engine/model_parallel/
token_dispatch.py:86-174`` (sort, count all-to-all + ``.tolist()``, three
variable all-to-alls, index_add), which this replaces on CUDA.
"""
from __future__ import annotations

import os

import torch
import torch.distributed as dist

from ...ops._ext import ext
from ...ops.moe import LocalExpertTransport, RoutePlan
from ...profiling import collective_profile
from ..comm.p2p import P2PSmallAllReduce, SymmBuffer, p2p_supported


class _RowPool:
    """Two rotating symmetric row buffers [rows_cap, H] bf16 of the EP group."""

    def __init__(self, group, device, rows_cap: int, hidden: int):
        self.rows_cap, self.hidden = rows_cap, hidden
        self.sets = [SymmBuffer(rows_cap * hidden, torch.bfloat16, device, group, "ep_rows") for _ in range(2)]
        self.turn = 0

    def next(self) -> SymmBuffer:
        buf = self.sets[self.turn % 2]
        self.turn += 1
        return buf


class PeerExpertTransport(LocalExpertTransport):
    """Routes of this rank's tokens to the owners of their experts over the
    EP group's peer memory (see module docstring)."""

    def __init__(self, partition, group, device):
        super().__init__(partition.local_count, num_experts=partition.num_experts, ep_rank=dist.get_rank(group))
        self.partition = partition
        self.group = group
        self.world = dist.get_world_size(group)
        self.device = device
        self.limit_s = float(os.environ.get("PB_P2P_TIMEOUT_S", "60"))
        self.pool: _RowPool | None = None
        self.small = P2PSmallAllReduce.get(group, device)

    @staticmethod
    def available(group, device) -> bool:
        return device.type == "cuda" and p2p_supported(group)

    # ------------------------------------------------------------------ plan
    def routes_in(self, routes: int) -> int:
        return routes * self.world  # every rank's routes could pick this owner

    def _histogram(self, topi: torch.Tensor, num_experts: int):
        mat = torch.empty(self.world, num_experts, dtype=torch.float32, device=topi.device)
        ext().moe_hist(topi, mat, self.ep_rank)
        flat = mat.view(-1)
        with collective_profile("ep_all_reduce", value=flat, mode="p2p" if self.small else "nccl",
                                detail="route_histograms"):
            if self.small is not None and flat.numel() <= 3 * self.small.cap:
                self.small.all_reduce_(flat)
            else:
                dist.all_reduce(flat, op=dist.ReduceOp.SUM, group=self.group)
        return mat, self.ep_rank

    def _rows(self, plan: RoutePlan, hidden: int) -> _RowPool:
        if self.pool is None:
            self.pool = _RowPool(self.group, self.device, plan.rows_cap, hidden)
        elif plan.rows_cap > self.pool.rows_cap or hidden != self.pool.hidden:
            raise RuntimeError(f"expert exchange buffers hold {self.pool.rows_cap} rows x {self.pool.hidden}; this "
                               f"layer needs {plan.rows_cap} x {hidden} (the token count per rank must stay fixed)")
        return self.pool

    def _barrier(self, buf: SymmBuffer) -> None:
        buf.barrier(0, self.limit_s)

    # ------------------------------------------------------------------ forward
    def dispatch(self, x2: torch.Tensor, plan: RoutePlan) -> torch.Tensor:
        H = x2.shape[1]
        recv = self._rows(plan, H).next()
        with collective_profile("ep_dispatch", value=x2, mode="p2p", detail="routes"):
            ext().moe_dispatch(x2, plan.top_k, plan.route_owner, plan.route_row, list(recv.peer_ptrs), H)
            self._barrier(recv)
        x_pad = torch.empty(plan.rows_cap, H, device=x2.device, dtype=x2.dtype)
        self._pad(recv.tensor.data_ptr(), H, x_pad, plan)
        return x_pad

    def output_buffer(self, plan: RoutePlan, H: int, like: torch.Tensor):
        send = self._rows(plan, H).next()
        return send.tensor[: plan.rows_cap * H].view(plan.rows_cap, H), send

    def combine(self, handle: SymmBuffer, plan: RoutePlan, weights, out, keep) -> None:
        with collective_profile("ep_combine", value=out, mode="p2p", detail="routes"):
            self._barrier(handle)
            ext().moe_combine(out, keep, weights, plan.route_owner, plan.route_row, list(handle.peer_ptrs),
                              out.shape[1])

    # ------------------------------------------------------------------ backward
    def combine_backward(self, dout, keep, weights, plan: RoutePlan):
        H = dout.shape[1]
        recv = self._rows(plan, H).next()
        dw = torch.empty(weights.shape, device=dout.device, dtype=torch.float32)
        with collective_profile("ep_combine", value=dout, mode="p2p_grad", detail="routes"):
            ext().moe_combine_bwd(dout, keep, weights, plan.route_owner, plan.route_row, list(recv.peer_ptrs), H, dw)
            self._barrier(recv)
        dy_pad = torch.empty(plan.rows_cap, H, device=dout.device, dtype=dout.dtype)
        self._pad(recv.tensor.data_ptr(), H, dy_pad, plan)
        return dy_pad, dw

    def grad_buffer(self, plan: RoutePlan, H: int, like: torch.Tensor):
        return self.output_buffer(plan, H, like)

    def gather_grad(self, handle: SymmBuffer, plan: RoutePlan, dx: torch.Tensor) -> None:
        with collective_profile("ep_dispatch", value=dx, mode="p2p_grad", detail="routes"):
            self._barrier(handle)
            ext().moe_combine(dx, None, None, plan.route_owner, plan.route_row, list(handle.peer_ptrs), dx.shape[1])
