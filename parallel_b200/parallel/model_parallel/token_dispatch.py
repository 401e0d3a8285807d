"""Variable-size all-to-all routing of top-k token routes to expert owners.

Dispatch sorts routes by owning rank (stable), exchanges per-rank counts,
then sends hidden rows, local expert ids and scores with variable-split
all-to-alls; combine returns expert outputs and sums them onto their source
tokens.  The autograd backward of every exchange is the reversed exchange.
Reference semantics: parallel/parallel/engine/model_parallel/token_dispatch.py.
"""
from __future__ import annotations

from dataclasses import dataclass

import torch
import torch.distributed as dist

from ...profiling import collective_profile


class _VariableAllToAll(torch.autograd.Function):
    @staticmethod
    def forward(ctx, value, send_splits, recv_splits, group, mode, detail):
        ctx.send, ctx.recv, ctx.group, ctx.mode, ctx.detail = tuple(send_splits), tuple(recv_splits), group, mode, detail
        out = torch.empty((sum(ctx.recv), *value.shape[1:]), dtype=value.dtype, device=value.device)
        with collective_profile("ep_all_to_all", value=value, mode=mode, detail=detail):
            dist.all_to_all_single(out, value.contiguous(), output_split_sizes=list(ctx.recv),
                                   input_split_sizes=list(ctx.send), group=group)
        return out

    @staticmethod
    def backward(ctx, g):
        out = torch.empty((sum(ctx.send), *g.shape[1:]), dtype=g.dtype, device=g.device)
        with collective_profile("ep_all_to_all", value=g, mode=f"{ctx.mode}_grad", detail=ctx.detail):
            dist.all_to_all_single(out, g.contiguous(), output_split_sizes=list(ctx.send),
                                   input_split_sizes=list(ctx.recv), group=ctx.group)
        return out, None, None, None, None, None


def variable_all_to_all(value, send_splits, receive_splits, group, *, mode="", detail=""):
    return _VariableAllToAll.apply(value, send_splits, receive_splits, group, mode, detail)


@dataclass
class DispatchState:
    send_splits: tuple
    receive_splits: tuple
    source_tokens: torch.Tensor
    num_source_tokens: int


class TokenDispatcher:
    """Dispatch routes to expert owners and restore source-token order."""

    def __init__(self, partition, group):
        self.partition = partition
        self.group = group
        self.world_size = dist.get_world_size(group)

    def _exchange_splits(self, destinations: torch.Tensor):
        send = torch.bincount(destinations, minlength=self.world_size).to(torch.int64)
        recv = torch.empty_like(send)
        with collective_profile("ep_all_to_all", value=send, mode="split_counts", detail="route_counts"):
            dist.all_to_all_single(recv, send, group=self.group)
        both = torch.stack([send, recv]).tolist()
        return tuple(both[0]), tuple(both[1])

    def dispatch(self, hidden_states, global_indices, scores):
        if global_indices.shape != scores.shape:
            raise ValueError("Expert indices and scores must have the same shape")
        tokens, top_k = global_indices.shape
        flat_e = global_indices.reshape(-1)
        flat_s = scores.reshape(-1)
        src = torch.arange(tokens, device=hidden_states.device).unsqueeze(1).expand(tokens, top_k).reshape(-1)
        dest = self.partition.owner(flat_e)
        order = torch.argsort(dest, stable=True)
        dest = dest[order]
        src = src[order]
        send_splits, recv_splits = self._exchange_splits(dest)
        send_hidden = hidden_states.index_select(0, src)
        send_experts = flat_e[order] - dest * self.partition.local_count
        send_scores = flat_s[order]
        rh = variable_all_to_all(send_hidden, send_splits, recv_splits, self.group, mode="dispatch_hidden",
                                 detail="routes")
        re = variable_all_to_all(send_experts, send_splits, recv_splits, self.group, mode="dispatch_experts",
                                 detail="routes")
        rs = variable_all_to_all(send_scores, send_splits, recv_splits, self.group, mode="dispatch_scores",
                                 detail="routes")
        return rh, re.unsqueeze(-1), rs.unsqueeze(-1), DispatchState(send_splits, recv_splits, src, tokens)

    def combine(self, expert_output: torch.Tensor, state: DispatchState):
        back = variable_all_to_all(expert_output, state.receive_splits, state.send_splits, self.group,
                                   mode="combine_hidden", detail="routes")
        out = torch.zeros((state.num_source_tokens, *back.shape[1:]), dtype=back.dtype, device=back.device)
        return out.index_add(0, state.source_tokens, back)
