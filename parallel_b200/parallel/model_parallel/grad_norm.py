"""Distributed gradient norm and clipping for model-parallel training.

Replicated parameters (shard_dim None) are counted on TP rank 0 only; the
squared sum is all-reduced over TP and then over the dp_shard group
(reference: parallel/parallel/engine/model_parallel/grad_norm.py:15-82).
"""
from __future__ import annotations

import torch
import torch.distributed as dist

from ...profiling import collective_profile
from ...state import Strategies
from .plan import ModelParallelPlan


def _local(t):
    return t._local_tensor if hasattr(t, "_local_tensor") else t


def global_grad_norm(named_parameters, *, plan: ModelParallelPlan, tp_mesh, pconfig, device) -> torch.Tensor:
    sq = torch.zeros((), dtype=torch.float32, device=device)
    tp_rank = tp_mesh.get_local_rank()
    for name, p in named_parameters:
        if p.grad is None:
            continue
        if plan.placement_for_parameter(name).shard_dim is None and tp_rank != 0:
            continue
        sq += _local(p.grad).detach().float().pow(2).sum().to(device)
    with collective_profile("tp_all_reduce", value=sq, mode="grad_norm", detail="global_norm"):
        dist.all_reduce(sq, op=dist.ReduceOp.SUM, group=tp_mesh.get_group())
    if pconfig.dp_shard_size > 1:
        with collective_profile("fsdp_all_reduce", value=sq, mode="grad_norm", detail="global_norm"):
            dist.all_reduce(sq, op=dist.ReduceOp.SUM, group=pconfig.group(Strategies.DP_SHARD))
    return sq.sqrt()


def clip_grad_norm_(named_parameters, max_norm: float, *, plan, tp_mesh, pconfig, device) -> torch.Tensor:
    named_parameters = tuple(named_parameters)
    total = global_grad_norm(named_parameters, plan=plan, tp_mesh=tp_mesh, pconfig=pconfig, device=device)
    coef = torch.clamp(max_norm / (total + 1e-6), max=1.0)
    for _, p in named_parameters:
        if p.grad is not None:
            g = _local(p.grad)
            g.mul_(coef.to(g.device, g.dtype))
    return total
