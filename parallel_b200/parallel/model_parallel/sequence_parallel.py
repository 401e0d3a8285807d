"""Megatron-style sequence parallelism over the TP group.

Residual activations stay token-sharded (dim 1) between blocks; attention,
the dense MLP and the LM head see the gathered sequence; row-parallel
outputs are reduce-scattered.  The model inserts these collectives itself
(``models/qwen3.py`` DecoderLayer.forward) once ``SequenceParallelRuntime``
has switched its context to SP mode - the reference does the same with
forward pre-hooks (parallel/parallel/engine/model_parallel/
sequence_parallel.py:161-218).

Also the SP-global Switch auxiliary loss (double softmax included,
reference :239-280).
"""
from __future__ import annotations

import torch
import torch.distributed as dist

from ...profiling import collective_profile
from . import comm_ops


def gather_sequence(value: torch.Tensor, group, dim: int = 1) -> torch.Tensor:
    return comm_ops._GatherSeq.apply(value, group, dim)


def reduce_scatter_sequence(value: torch.Tensor, group, dim: int = 1) -> torch.Tensor:
    return comm_ops._ReduceScatterSeq.apply(value, group, dim)


def scatter_sequence(value: torch.Tensor, group, dim: int = 1) -> torch.Tensor:
    return comm_ops._ScatterSeq.apply(value, group, dim)


class SequenceParallelRuntime:
    """Switches the model's parallel context to sequence-parallel mode."""

    def __init__(self, group, *, dense_mlp: bool):
        self.group = group
        self.dense_mlp = dense_mlp
        self._model = None

    def apply(self, model) -> None:
        if self._model is not None:
            raise RuntimeError("Sequence-parallel runtime is already installed")
        layers = list(model.model.layers)
        if not layers:
            raise RuntimeError("sequence parallelism found no decoder layers in the model")
        ctx = model.ctx
        ctx.sp = True
        model.set_parallel_context(ctx)
        self._model = model

    def close(self) -> None:
        if self._model is not None:
            ctx = self._model.ctx
            ctx.sp = False
            self._model.set_parallel_context(ctx)
            self._model = None


class _AllReduceForwardIdentityBackward(torch.autograd.Function):
    """SUM over the group in forward, identity in backward (the reference's
    semantics for the SP router-probability sums).  ``small`` (a
    P2PSmallAllReduce) runs it as one peer-memory kernel instead of NCCL."""

    @staticmethod
    def forward(ctx, value, group, small=None):
        out = value.contiguous().clone()
        with collective_profile("sp_all_reduce", value=out, mode="router_statistics", detail="load_balancing_loss"):
            if small is not None:
                small.all_reduce_(out, "sum")
            else:
                dist.all_reduce(out, group=group)
        return out

    @staticmethod
    def backward(ctx, g):
        return g, None, None


def sequence_parallel_load_balancing_loss(router_logits, *, num_experts: int, top_k: int, group,
                                          collectives: str = "auto"):
    """Switch aux loss over the SP-global token population.  The per-expert
    top-k counts, the sums of softmax(probs) and the token count travel in
    one all-reduce (one peer-memory kernel on CUDA with NVLink), where the
    reference issues three (sequence_parallel.py:239-280)."""
    if not router_logits:
        return None
    from ...ops.moe import aux_loss_stats

    logits = torch.cat(tuple(router_logits), dim=0)
    # per-expert top-k counts and sums of softmax(probs) (one fused kernel on CUDA)
    counts, prob_sum = aux_loss_stats(logits.float(), top_k)
    ntok = torch.full((1,), float(logits.shape[0]), dtype=torch.float32, device=logits.device)
    small = None
    if collectives != "nccl" and logits.is_cuda:
        from ..comm.p2p import P2PSmallAllReduce

        small = P2PSmallAllReduce.get(group, logits.device)
    E = counts.numel()
    packed = _AllReduceForwardIdentityBackward.apply(torch.cat([counts.detach(), prob_sum, ntok]), group, small)
    counts, prob_sum, ntok = packed[:E], packed[E:2 * E], packed[2 * E]
    return num_experts * torch.sum((counts.detach() / ntok.detach()) * (prob_sum / ntok.detach()))
