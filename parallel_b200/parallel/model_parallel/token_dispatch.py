"""Expert-parallel token exchange through ``torch.distributed`` all-to-alls.

This is the portable path (CPU / gloo, or ``engine.collectives=nccl``); on
CUDA with NVLink peer access the SP expert parallelism runs on
``p2p_dispatch.PeerExpertTransport`` instead, which needs no host sync.

Behaviour of the reference's ``parallel/parallel/engine/model_parallel/
token_dispatch.py:11-174``: a rank's routes are grouped by owning rank
(stable, so each rank's routes keep their flat token-major order), the
per-owner counts are exchanged and read on the host (they are the split
sizes of the variable all-to-alls), hidden rows, local expert ids and
routing weights travel to the owners, and the owners' outputs travel back
and are summed onto their source tokens.  Organisation here:

* ``ExchangePlan`` holds one dispatch's split sizes and the source token of
  every sent row;
* ``_Exchange`` is the one autograd node of a variable all-to-all; its
  backward is the same exchange with the splits swapped.
"""
from __future__ import annotations

from dataclasses import dataclass

import torch
import torch.distributed as dist

from ...profiling import collective_profile


@dataclass
class ExchangePlan:
    send: list          # rows this rank sends to each owner
    recv: list          # rows this rank receives from each source
    source_tokens: torch.Tensor  # token of every sent row, in send order
    num_source_tokens: int

    # names the reference's dispatch state used
    @property
    def send_splits(self):
        return tuple(self.send)

    @property
    def receive_splits(self):
        return tuple(self.recv)


DispatchState = ExchangePlan


def _all_to_all(rows: torch.Tensor, out_splits, in_splits, group, mode: str) -> torch.Tensor:
    out = rows.new_empty((sum(out_splits), *rows.shape[1:]))
    with collective_profile("ep_all_to_all", value=rows, mode=mode, detail="routes"):
        dist.all_to_all_single(out, rows.contiguous(), output_split_sizes=list(out_splits),
                               input_split_sizes=list(in_splits), group=group)
    return out


class _Exchange(torch.autograd.Function):
    @staticmethod
    def forward(ctx, rows, send, recv, group, mode):
        ctx.send, ctx.recv, ctx.group, ctx.mode = send, recv, group, mode
        return _all_to_all(rows, recv, send, group, mode)

    @staticmethod
    def backward(ctx, grad):
        return _all_to_all(grad, ctx.send, ctx.recv, ctx.group, ctx.mode + "_grad"), None, None, None, None


def variable_all_to_all(value, send_splits, receive_splits, group, *, mode="", detail=""):
    """Differentiable variable-split all-to-all (rows along dim 0)."""
    return _Exchange.apply(value, list(send_splits), list(receive_splits), group, mode)


class TokenDispatcher:
    """Route rows to expert owners and back with all-to-alls (see module docstring)."""

    def __init__(self, partition, group):
        self.partition = partition
        self.group = group
        self.world_size = dist.get_world_size(group)

    def plan(self, owners_sorted: torch.Tensor, source_tokens: torch.Tensor, num_tokens: int) -> ExchangePlan:
        sent = torch.bincount(owners_sorted, minlength=self.world_size)
        got = torch.empty_like(sent)
        with collective_profile("ep_all_to_all", value=sent, mode="split_counts", detail="route_counts"):
            dist.all_to_all_single(got, sent, group=self.group)
        send, recv = torch.stack([sent, got]).tolist()  # the split sizes must be host integers
        return ExchangePlan(send, recv, source_tokens, num_tokens)

    def dispatch(self, hidden_states, global_indices, scores):
        """Returns (rows [R, H], local expert ids [R, 1], weights [R, 1], plan)."""
        if global_indices.shape != scores.shape:
            raise ValueError(f"expert ids {tuple(global_indices.shape)} and routing weights "
                             f"{tuple(scores.shape)} must have the same shape")
        tokens, k = global_indices.shape
        flat = global_indices.reshape(-1)
        owners = self.partition.owner(flat)
        by_owner = torch.sort(owners, stable=True).indices
        source = by_owner // k
        plan = self.plan(owners[by_owner], source, tokens)
        local_ids = (flat - owners * self.partition.local_count)[by_owner]
        rows = _Exchange.apply(hidden_states.index_select(0, source), plan.send, plan.recv, self.group,
                               "dispatch_hidden")
        with torch.no_grad():
            ids = _all_to_all(local_ids, plan.recv, plan.send, self.group, "dispatch_experts")
        weights = _Exchange.apply(scores.reshape(-1)[by_owner], plan.send, plan.recv, self.group, "dispatch_scores")
        return rows, ids.unsqueeze(-1), weights.unsqueeze(-1), plan

    def combine(self, expert_output: torch.Tensor, plan: ExchangePlan):
        """Owners' outputs back to the source ranks, summed per token."""
        back = _Exchange.apply(expert_output, plan.recv, plan.send, self.group, "combine_hidden")
        out = back.new_zeros((plan.num_source_tokens, *back.shape[1:]))
        return out.index_add(0, plan.source_tokens, back)
