"""Differentiable TP / SP collectives used inside the model.

Semantics (the mirror pairs of Megatron-style TP/SP, as in the HF styles the
reference installs, transformers/integrations/tensor_parallel.py, and in
parallel/parallel/engine/model_parallel/sequence_parallel.py:48-158):

* ``copy_to_tp``             identity fwd / all-reduce bwd  (column-parallel input)
* ``reduce_from_tp``         all-reduce fwd / identity bwd  (row-parallel output, vocab embedding)
* ``gather_sequence``        all-gather(dim 1) fwd / reduce-scatter bwd
* ``reduce_scatter_sequence`` reduce-scatter(dim 1) fwd / all-gather bwd
* ``scatter_sequence``       split(dim 1) fwd / all-gather bwd

Each takes the model's ``ParallelContext``; the data plane is torch.distributed
(NCCL on GPUs, gloo on CPU), except that the all-reduces of non-SP tensor
parallelism go over NVLink peer memory when the context carries a
``FusedTensorParallel`` (bf16 tensors whose rows divide over the group).
"""
from __future__ import annotations

import torch
import torch.distributed as dist

from ...profiling import collective_profile


def _front(t: torch.Tensor, dim: int) -> torch.Tensor:
    dim = dim if dim >= 0 else t.ndim + dim
    return t.movedim(dim, 0).contiguous()


def _back(t: torch.Tensor, dim: int, ndim: int) -> torch.Tensor:
    dim = dim if dim >= 0 else ndim + dim
    return t.movedim(0, dim).contiguous()


def all_gather_dim(value: torch.Tensor, group, dim: int, op_name: str = "sp_all_gather") -> torch.Tensor:
    world = dist.get_world_size(group)
    if world == 1:
        return value
    front = _front(value, dim)
    out = torch.empty((front.shape[0] * world, *front.shape[1:]), dtype=front.dtype, device=front.device)
    with collective_profile(op_name, value=front, mode="sequence", detail=f"shape={tuple(front.shape)}"):
        dist.all_gather_into_tensor(out, front, group=group)
    return _back(out, dim, value.ndim)


def reduce_scatter_dim(value: torch.Tensor, group, dim: int, op_name: str = "sp_reduce_scatter") -> torch.Tensor:
    world = dist.get_world_size(group)
    if world == 1:
        return value
    d = dim if dim >= 0 else value.ndim + dim
    if value.shape[d] % world:
        raise ValueError(f"Sequence dimension {value.shape[d]} must be divisible by sequence-parallel size {world}")
    front = _front(value, dim)
    out = torch.empty((front.shape[0] // world, *front.shape[1:]), dtype=front.dtype, device=front.device)
    with collective_profile(op_name, value=front, mode="sequence", detail=f"shape={tuple(front.shape)}"):
        dist.reduce_scatter_tensor(out, front, op=dist.ReduceOp.SUM, group=group)
    return _back(out, dim, value.ndim)


def all_reduce_sum(value: torch.Tensor, group, op_name: str = "tp_all_reduce", mode: str = "",
                   fused=None) -> torch.Tensor:
    """SUM over ``group``; ``fused`` (a FusedTensorParallel) runs it over NVLink
    peer memory when the tensor fits its buffers, NCCL / gloo otherwise."""
    if fused is not None:
        out = fused.try_all_reduce(value)
        if out is not None:
            return out
    out = value.contiguous().clone()
    with collective_profile(op_name, value=out, mode=mode):
        dist.all_reduce(out, op=dist.ReduceOp.SUM, group=group)
    return out


class _CopyToTP(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, group, fused):
        ctx.group, ctx.fused = group, fused
        return x

    @staticmethod
    def backward(ctx, g):
        return all_reduce_sum(g, ctx.group, mode="colwise_input_grad", fused=ctx.fused), None, None


class _ReduceFromTP(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, group, fused):
        return all_reduce_sum(x, group, mode="rowwise_output", fused=fused)

    @staticmethod
    def backward(ctx, g):
        return g, None, None


def _p2p_all_reduce(ctx):
    """The context's NVLink all-reduce (FusedTensorParallel, non-SP TP) or None."""
    f = getattr(ctx, "fused_tp", None)
    return f if f is not None and hasattr(f, "try_all_reduce") else None


class _GatherSeq(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, group, dim):
        ctx.group, ctx.dim = group, dim
        return all_gather_dim(x, group, dim)

    @staticmethod
    def backward(ctx, g):
        return reduce_scatter_dim(g, ctx.group, ctx.dim), None, None


class _ReduceScatterSeq(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, group, dim):
        ctx.group, ctx.dim = group, dim
        return reduce_scatter_dim(x, group, dim)

    @staticmethod
    def backward(ctx, g):
        return all_gather_dim(g, ctx.group, ctx.dim), None, None


class _ScatterSeq(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, group, dim):
        ctx.group, ctx.dim = group, dim
        world = dist.get_world_size(group)
        rank = dist.get_rank(group)
        d = dim if dim >= 0 else x.ndim + dim
        if x.shape[d] % world:
            raise ValueError(f"Sequence dimension {x.shape[d]} must be divisible by sequence-parallel size {world}")
        return x.chunk(world, dim=d)[rank].contiguous()

    @staticmethod
    def backward(ctx, g):
        return all_gather_dim(g, ctx.group, ctx.dim), None, None


def copy_to_tp(x, ctx):
    return _CopyToTP.apply(x, ctx.tp_group, _p2p_all_reduce(ctx))


def reduce_from_tp(x, ctx):
    return _ReduceFromTP.apply(x, ctx.tp_group, _p2p_all_reduce(ctx))


def gather_sequence(x, ctx, dim: int = 1):
    return _GatherSeq.apply(x, ctx.tp_group, dim)


def reduce_scatter_sequence(x, ctx, dim: int = 1):
    return _ReduceScatterSeq.apply(x, ctx.tp_group, dim)


def scatter_sequence(x, ctx, dim: int = 1):
    return _ScatterSeq.apply(x, ctx.tp_group, dim)
