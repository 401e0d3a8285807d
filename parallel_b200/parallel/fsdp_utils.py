"""Helpers shared by the FSDP engine (reference: parallel/parallel/engine/_dp_sharded_utils.py)."""
from __future__ import annotations

import torch
import torch.nn as nn
from torch.distributed.tensor import DTensor


def group_named_parameters(named_parameters):
    """Split into groups of equal (device, dtype, requires_grad), keeping order."""
    groups: dict = {}
    for name, p in named_parameters:
        groups.setdefault((p.device, p.dtype, p.requires_grad), []).append((name, p))
    return list(groups.values())


def get_fsdp_units(model: nn.Module) -> list[nn.Module]:
    """Decoder layers are the FSDP units (``model.model.layers`` for causal LMs)."""
    if hasattr(model, "model") and hasattr(model.model, "layers"):
        return list(model.model.layers)
    if hasattr(model, "transformer") and hasattr(model.transformer, "h"):
        return list(model.transformer.h)
    if hasattr(model, "layers"):
        return list(model.layers)
    return [model]


def discover_used_parameter_ids(loss: torch.Tensor, parameter_ids: set[int]) -> set[int]:
    """Leaf parameters reachable from ``loss``'s autograd graph."""
    used: set[int] = set()
    if id(loss) in parameter_ids:
        used.add(id(loss))
    if loss.grad_fn is None:
        return used
    stack, seen = [loss.grad_fn], set()
    while stack:
        node = stack.pop()
        if node in seen:
            continue
        seen.add(node)
        var = getattr(node, "variable", None)
        if var is not None and id(var) in parameter_ids:
            used.add(id(var))
        for nxt, _ in node.next_functions:
            if nxt is not None:
                stack.append(nxt)
    return used


def local_tensor(t: torch.Tensor) -> torch.Tensor:
    return t._local_tensor if isinstance(t, DTensor) else t
