"""Tensor-parallel mesh, model verification and SUM_TP gradient reductions.

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
        raise RuntimeError("tensor parallelism needs the device mesh (set_device_mesh first)")
    if mesh.ndim == 1:
        return mesh
    if Strategies.TP.value not in mesh.mesh_dim_names:
        raise RuntimeError("the device mesh has no 'tp' dimension")
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
    if device is not None and torch.device(device).type == "cuda":
        # built, drawn and cast on the GPU: a 30B-class model's local shards
        # never pass through host memory
        prev = torch.get_default_dtype()
        torch.set_default_dtype(dtype)
        try:
            with torch.device(device):
                model = Qwen3ForCausalLM(config, tp=tp, ep=ep)
        finally:
            torch.set_default_dtype(prev)
    else:
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


def install_tensor_parallel_gradient_hooks(model, plan: ModelParallelPlan, tp_mesh, exclude=frozenset()):
    """All-reduce (sum) the partial gradients of SUM_TP replicated params, one
    collective per parameter (parallel/parallel/engine/model_parallel/
    tensor_parallel.py:121-141); ``exclude`` names the params whose sums a
    per-layer ``LayerGradientPack`` does instead."""
    handles = []
    group = tp_mesh.get_group()

    def hook(g):
        out = g.contiguous().clone()
        with collective_profile("tp_all_reduce", value=out, mode="replicated_param_grad", detail="parameter_hook"):
            dist.all_reduce(out, op=dist.ReduceOp.SUM, group=group)
        return out

    for name, p in model.named_parameters():
        if name in exclude:
            continue
        if plan.placement_for_parameter(name).gradient_reduction == GradientReduction.SUM_TP:
            handles.append(p.register_hook(hook))
    return handles


class _PackedGradSum(torch.autograd.Function):
    """Identity on a layer's SUM_TP parameters in forward.  Autograd runs the
    backward once every use of them in the layer has produced its gradient, so
    all their partial gradients arrive together and are summed over the TP
    group in ONE collective."""

    @staticmethod
    def forward(ctx, pack, *params):
        ctx.pack = pack
        return tuple(p.view_as(p) for p in params)

    @staticmethod
    def backward(ctx, *grads):
        return (None,) + ctx.pack.reduce(grads)


class LayerGradientPack:
    """The SUM_TP parameters of one decoder layer (q_norm and k_norm; under
    sequence parallelism also both layer norms and the MoE router).  The
    reference sums each one over TP in its own all-reduce from a parameter
    hook (4-5 per layer); here the layer's forward runs with its parameters
    routed through ``_PackedGradSum``, and their gradients are summed as one
    fp32 vector: on CUDA over NVLink with ``P2PSmallAllReduce`` when the vector
    fits its buffer (the layer norms and q/k-norms of every benchmark model),
    with a single NCCL / gloo all-reduce otherwise (e.g. a 128 x 2048 router).
    The sums are the reference's, accumulated in fp32 instead of the grads'
    dtype."""

    def __init__(self, layer, rel_names: list[str], group, small=None):
        self.group = group
        self.small = small
        self.rel_names = list(rel_names)
        self.slots = []
        for rel in self.rel_names:
            mod_path, _, leaf = rel.rpartition(".")
            self.slots.append((layer.get_submodule(mod_path) if mod_path else layer, leaf))
        self.numel = sum(getattr(m, leaf).numel() for m, leaf in self.slots)

    def run(self, layer_forward, *args):
        """Call ``layer_forward(*args)`` with the layer's SUM_TP parameters
        replaced by ``_PackedGradSum`` views of themselves."""
        params = [m._parameters[leaf] for m, leaf in self.slots]
        views = _PackedGradSum.apply(self, *params)
        for (m, leaf), v in zip(self.slots, views):
            m._parameters[leaf] = v
        try:
            return layer_forward(*args)
        finally:
            for (m, leaf), p in zip(self.slots, params):
                m._parameters[leaf] = p

    def reduce(self, grads) -> tuple:
        ref = next((g for g in grads if g is not None), None)
        if ref is None:
            return (None,) * len(grads)
        parts = []
        for (m, leaf), g in zip(self.slots, grads):
            n = m._parameters[leaf].numel()
            parts.append(g.reshape(-1).float() if g is not None else torch.zeros(n, device=ref.device))
        flat = torch.cat(parts)
        with collective_profile("tp_all_reduce", value=flat, mode="replicated_param_grad", detail="layer_packed"):
            if self.small is not None and flat.is_cuda and flat.numel() <= 3 * self.small.cap:
                self.small.all_reduce_(flat)
            else:
                dist.all_reduce(flat, op=dist.ReduceOp.SUM, group=self.group)
        out, o = [], 0
        for g, part in zip(grads, parts):
            n = part.numel()
            out.append(None if g is None else flat[o:o + n].view(g.shape).to(g.dtype))
            o += n
        return tuple(out)


def install_layer_gradient_packs(model, plan: ModelParallelPlan, tp_mesh, small=None) -> set[str]:
    """Give every decoder layer with SUM_TP parameters a ``LayerGradientPack``
    (``layer._tp_grad_pack``); returns the names it covers (their per-param
    hooks are not installed)."""
    group = tp_mesh.get_group()
    covered: set[str] = set()
    layers = getattr(getattr(model, "model", None), "layers", None)
    if layers is None:
        return covered
    for i, layer in enumerate(layers):
        prefix = f"model.layers.{i}."
        rel = [n for n, _ in layer.named_parameters()
               if plan.placement_for_parameter(prefix + n).gradient_reduction == GradientReduction.SUM_TP]
        if rel:
            layer._tp_grad_pack = LayerGradientPack(layer, rel, group, small)
            covered.update(prefix + n for n in rel)
    return covered
