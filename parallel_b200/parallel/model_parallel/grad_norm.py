"""Global gradient norm and clipping of a model-parallel (optionally FSDP) model.

The norm is sqrt(sum_i w_i * ||g_i||^2) over the rank-local gradient shards,
summed over the TP group and then over the dp_shard group.  ``w_i`` is 1 for
a parameter sharded over TP and, for a parameter replicated over TP (plan
``shard_dim`` None), 1 on TP rank 0 and 0 elsewhere, so every replicated
gradient counts once (reference behaviour,
``parallel/parallel/engine/model_parallel/grad_norm.py:15-82``).  The CUDA
training step computes the same weighted sum in one multi-tensor kernel
(``ParallelEngine._grad_lists``); this module is the generic path (CPU,
fp16 loss scaling).  Clip coefficient: min(1, max_norm / (norm + 1e-6)).
"""
from __future__ import annotations

import torch
import torch.distributed as dist

from ...profiling import collective_profile
from ...state import Strategies
from ..fsdp_utils import local_tensor
from .plan import ModelParallelPlan


def norm_weights(named_parameters, plan: ModelParallelPlan, tp_rank: int):
    """(local gradient, weight) of every parameter that has a gradient."""
    for name, param in named_parameters:
        if param.grad is None:
            continue
        replicated = plan.placement_for_parameter(name).shard_dim is None
        yield local_tensor(param.grad), (0.0 if (replicated and tp_rank != 0) else 1.0)


def _weighted_square_sum(pairs, device) -> torch.Tensor:
    total = torch.zeros((), dtype=torch.float32, device=device)
    for grad, weight in pairs:
        if weight:
            total += torch.linalg.vector_norm(grad.detach(), dtype=torch.float32).to(device).square() * weight
    return total


def _reduce_over(total: torch.Tensor, pconfig, tp_group) -> torch.Tensor:
    stages = [("tp_all_reduce", tp_group)]
    if pconfig.dp_shard_size > 1:
        stages.append(("fsdp_all_reduce", pconfig.group(Strategies.DP_SHARD)))
    for op, group in stages:
        with collective_profile(op, value=total, mode="grad_norm", detail="global_norm"):
            dist.all_reduce(total, op=dist.ReduceOp.SUM, group=group)
    return total


def global_grad_norm(named_parameters, *, plan: ModelParallelPlan, tp_mesh, pconfig, device) -> torch.Tensor:
    pairs = norm_weights(named_parameters, plan, tp_mesh.get_local_rank())
    return _reduce_over(_weighted_square_sum(pairs, device), pconfig, tp_mesh.get_group()).sqrt()


def clip_grad_norm_(named_parameters, max_norm: float, *, plan, tp_mesh, pconfig, device) -> torch.Tensor:
    """Scale every local gradient by the clip coefficient; returns the norm."""
    named_parameters = list(named_parameters)
    norm = global_grad_norm(named_parameters, plan=plan, tp_mesh=tp_mesh, pconfig=pconfig, device=device)
    coefficient = (max_norm / (norm + 1e-6)).clamp(max=1.0)
    grads = [local_tensor(p.grad) for _, p in named_parameters if p.grad is not None]
    for grad in grads:
        grad.mul_(coefficient.to(device=grad.device, dtype=grad.dtype))
    return norm
