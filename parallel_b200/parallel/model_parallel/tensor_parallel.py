"""Tensor-parallel mesh, model verification and SUM_TP gradient hooks.

The reference loads HF models with ``tp_plan`` so every rank materialises
only its shards (parallel/parallel/engine/model_parallel/tensor_parallel.py).
Here the model classes are built with local shapes directly
(``models.qwen3.Qwen3ForCausalLM(config, tp=..., ep=...)``) and weights are
loaded by ``load_tensor_parallel_causal_lm`` from a portable state dict
(each rank slices its shard by the plan's ``shard_dim``).
"""
from __future__ import annotations

import os

import torch
import torch.distributed as dist

from ...profiling import collective_profile
from ...state import Strategies
from .plan import GradientReduction, ModelParallelPlan, ParameterParallelism


def tensor_parallel_mesh(pconfig):
    mesh = pconfig.device_mesh
    if mesh is None:
        raise RuntimeError("Tensor parallelism requires a DeviceMesh")
    if mesh.ndim == 1:
        return mesh
    if Strategies.TP.value not in mesh.mesh_dim_names:
        raise RuntimeError("The distributed DeviceMesh has no tp dimension")
    return mesh[Strategies.TP.value]


def shard_for_rank(full: torch.Tensor, placement, tp_size: int, tp_rank: int) -> torch.Tensor:
    """This rank's slice of a full tensor under ``placement``."""
    if placement.shard_dim is None or placement.parallelism == ParameterParallelism.REPLICATED:
        return full
    return full.chunk(tp_size, dim=placement.shard_dim)[tp_rank]


def load_tensor_parallel_causal_lm(model_name: str, *, config, pconfig, plan: ModelParallelPlan, dtype=torch.bfloat16,
                                   device=None, seed: int | None = None, **_):
    """Build the local-shape model; load this rank's shards from
    ``model_name`` (a directory with ``model.pt`` / ``pytorch_model.bin`` /
    ``*.safetensors``) or keep the random init when it has no weights."""
    from ...models.qwen3 import Qwen3ForCausalLM
    from ...models.loading import read_state_dict

    tp = plan.tensor_parallel_size
    ep = plan.expert_parallel_size
    model = Qwen3ForCausalLM(config, tp=tp, ep=ep)
    model.init_weights(seed=seed)
    model.to(dtype=dtype)
    full = read_state_dict(model_name) if model_name and os.path.isdir(model_name) else None
    mesh = tensor_parallel_mesh(pconfig)
    rank = mesh.get_local_rank()
    if full is not None:
        with torch.no_grad():
            for name, p in model.named_parameters():
                if name not in full:
                    continue
                pl = plan.placement_for_parameter(name)
                p.copy_(shard_for_rank(full[name], pl, tp, rank).to(p.dtype))
    if device is not None:
        model.to(device)
    model._layout_fused_weights()
    model._tp_size = tp
    verify_tensor_parallel_model(model, plan, mesh)
    return model


def verify_tensor_parallel_model(model, plan: ModelParallelPlan, tp_mesh) -> None:
    loaded = getattr(model, "_tp_size", getattr(model, "tp_size", None))
    if loaded != plan.tensor_parallel_size:
        raise RuntimeError(f"Expected loaded TP size {plan.tensor_parallel_size}, got {loaded}")
    params = dict(model.named_parameters())
    plan.validate_parameter_coverage(params)
    if tp_mesh.size() != plan.tensor_parallel_size:
        raise RuntimeError(f"TP mesh size {tp_mesh.size()} does not match plan size {plan.tensor_parallel_size}")
    if dist.is_initialized() and tp_mesh.size() > 1:
        group = tp_mesh.get_group()
        shapes = {n: tuple(p.shape) for n, p in params.items()}
        gathered = [None] * tp_mesh.size()
        dist.all_gather_object(gathered, shapes, group=group)
        for r, s in enumerate(gathered):
            if set(s) != set(shapes):
                raise RuntimeError(f"TP rank {r} has a different parameter set")
        for n in params:
            pl = plan.placement_for_parameter(n)
            ss = [g[n] for g in gathered]
            if any(x != ss[0] for x in ss[1:]):
                raise RuntimeError(f"Uneven or inconsistent TP shards for {n}: {ss}")
            if pl.shard_dim is not None and ss[0][pl.shard_dim] == 0:
                raise RuntimeError(f"Empty TP shard for {n}")


def install_tensor_parallel_gradient_hooks(model, plan: ModelParallelPlan, tp_mesh):
    """All-reduce (sum) the partial gradients of SUM_TP replicated params."""
    handles = []
    group = tp_mesh.get_group()

    def hook(g):
        out = g.contiguous().clone()
        with collective_profile("tp_all_reduce", value=out, mode="replicated_param_grad", detail="parameter_hook"):
            dist.all_reduce(out, op=dist.ReduceOp.SUM, group=group)
        return out

    for name, p in model.named_parameters():
        if plan.placement_for_parameter(name).gradient_reduction == GradientReduction.SUM_TP:
            handles.append(p.register_hook(hook))
    return handles
