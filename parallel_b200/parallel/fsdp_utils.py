"""Small helpers of the FSDP engine: unit discovery, parameter grouping,
DTensor local views and autograd-graph reachability.

Behaviour of the reference's ``parallel/parallel/engine/_dp_sharded_utils.py``
(which layers become units, how parameters are grouped into flat buckets).
"""
from __future__ import annotations

from itertools import groupby

import torch
import torch.nn as nn
from torch.distributed.tensor import DTensor

# attribute paths, tried in order, to a causal LM's list of decoder layers
_LAYER_PATHS = (("model", "layers"), ("transformer", "h"), ("layers",))


def get_fsdp_units(model: nn.Module) -> list[nn.Module]:
    """The modules that become FSDP units: the decoder layers, or the whole
    model when it has no recognisable layer list."""
    for path in _LAYER_PATHS:
        node = model
        for attr in path:
            node = getattr(node, attr, None)
            if node is None:
                break
        if node is not None:
            return list(node)
    return [model]


def group_named_parameters(named_parameters) -> list[list]:
    """Partition (name, parameter) pairs by (device, dtype, requires_grad):
    one flat bucket holds one kind only.  Groups appear in order of their
    first member and keep the members' order."""
    named_parameters = list(named_parameters)
    key = lambda item: (item[1].device, item[1].dtype, item[1].requires_grad)  # noqa: E731
    first_seen = {}
    for i, item in enumerate(named_parameters):
        first_seen.setdefault(key(item), i)
    ordered = sorted(named_parameters, key=lambda item: first_seen[key(item)])  # stable within a group
    return [list(members) for _, members in groupby(ordered, key=lambda item: first_seen[key(item)])]


def discover_used_parameter_ids(loss: torch.Tensor, parameter_ids: set[int]) -> set[int]:
    """Ids (from ``parameter_ids``) of the leaves ``loss`` depends on, found by
    walking its autograd graph from the output."""
    found = {id(loss)} & parameter_ids
    frontier = [loss.grad_fn] if loss.grad_fn is not None else []
    visited = set()
    while frontier:
        node = frontier.pop()
        if node is None or node in visited:
            continue
        visited.add(node)
        leaf = getattr(node, "variable", None)  # AccumulateGrad nodes hold the leaf
        if leaf is not None and id(leaf) in parameter_ids:
            found.add(id(leaf))
        frontier.extend(parent for parent, _ in node.next_functions)
    return found


def local_tensor(t: torch.Tensor) -> torch.Tensor:
    """The rank-local tensor behind a DTensor (the tensor itself otherwise)."""
    return t._local_tensor if isinstance(t, DTensor) else t
