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
            raise RuntimeError("Sequence parallelism requires decoder layers")
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
    @staticmethod
    def forward(ctx, value, group):
        out = value.contiguous().clone()
        with collective_profile("sp_all_reduce", value=out, mode="router_probability", detail="load_balancing_loss"):
            dist.all_reduce(out, group=group)
        return out

    @staticmethod
    def backward(ctx, g):
        return g, None


def sequence_parallel_load_balancing_loss(router_logits, *, num_experts: int, top_k: int, group):
    """Switch aux loss over the SP-global token population."""
    if not router_logits:
        return None
    from ...ops.moe import aux_loss_stats

    logits = torch.cat(tuple(router_logits), dim=0)
    # per-expert top-k counts and sums of softmax(probs) (one fused kernel on CUDA)
    counts, prob_sum = aux_loss_stats(logits.float(), top_k)
    ntok = torch.tensor(logits.shape[0], dtype=torch.float32, device=logits.device)
    with collective_profile("sp_all_reduce", value=counts, mode="router_counts", detail="load_balancing_loss"):
        dist.all_reduce(counts, group=group)
    with collective_profile("sp_all_reduce", value=ntok, mode="token_count", detail="load_balancing_loss"):
        dist.all_reduce(ntok, group=group)
    prob_sum = _AllReduceForwardIdentityBackward.apply(prob_sum, group)
    return num_experts * torch.sum((counts / ntok) * (prob_sum / ntok))
