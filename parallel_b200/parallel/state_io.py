"""Model state-dict plumbing shared by the FSDP wrapper and the model-parallel
checkpoint adapters.

Three objects can own a model's portable ("full") state dict: the FSDP
wrapper (flat units, dp_shard row shards), the model-parallel adapter (TP /
EP shards) and the composition of both.  They differ only in where a full
tensor comes from and where it goes; what a valid incoming state dict looks
like is the same question for all of them.  This module answers it once:

* ``StateCatalog`` lists the model's state-dict entries in order, each with
  the full shape an incoming dict must carry, whether it is a parameter, and
  the dimension tensor parallelism splits it along (``None`` = replicated);
* ``StateCatalog.audit`` checks an incoming dict against it and returns a
  ``LoadReport`` (missing / unexpected keys and problems), which the loading
  rank broadcasts so every rank raises or proceeds together;
* ``tp_assemble`` / ``tp_distribute`` join TP shards into a full tensor and
  split a full tensor back into TP shards, driven by the catalog's split
  dimension rather than per-method branches.

The reference's per-wrapper equivalents are
``parallel/parallel/engine/dp_sharded.py:556-868`` and
``parallel/parallel/engine/model_parallel/checkpoint.py:18-461``.
"""
from __future__ import annotations

import copy
from collections import OrderedDict
from dataclasses import dataclass, field
from typing import Any, Iterable, Optional

import torch
import torch.distributed as dist
import torch.nn as nn
from torch.distributed.tensor import DTensor


def host_tensor(value: Any) -> Any:
    """A detached CPU copy of a tensor (the local shard of a DTensor); other
    values are deep-copied."""
    if isinstance(value, DTensor):
        value = value._local_tensor
    if isinstance(value, torch.Tensor):
        return value.detach().to("cpu", copy=True)
    return copy.deepcopy(value)


def with_metadata(out: OrderedDict, source) -> OrderedDict:
    """Carry ``state_dict()._metadata`` (module versions) over to ``out``."""
    meta = getattr(source, "_metadata", None)
    if meta is not None:
        out._metadata = copy.deepcopy(meta)
    return out


@dataclass(frozen=True)
class Entry:
    name: str
    is_param: bool
    full_shape: Optional[tuple]      # None: not a tensor (no shape to check)
    dtype: Optional[torch.dtype]
    tp_dim: Optional[int] = None     # dim TP splits the tensor along


@dataclass
class LoadReport:
    missing: list = field(default_factory=list)
    unexpected: list = field(default_factory=list)
    problems: list = field(default_factory=list)
    present: list = field(default_factory=list)

    def raise_if_bad(self, what: str) -> None:
        if self.problems:
            raise RuntimeError(f"cannot load {what}: " + "; ".join(self.problems))

    def incompatible_keys(self):
        return nn.modules.module._IncompatibleKeys(self.missing, self.unexpected)


class StateCatalog:
    """Ordered description of the state dict a wrapper accepts (see module doc)."""

    def __init__(self, entries: Iterable[Entry]):
        self.entries: "OrderedDict[str, Entry]" = OrderedDict((e.name, e) for e in entries)

    def __iter__(self):
        return iter(self.entries.values())

    def __contains__(self, name: str) -> bool:
        return name in self.entries

    def __getitem__(self, name: str) -> Entry:
        return self.entries[name]

    def names(self) -> list[str]:
        return list(self.entries)

    def audit(self, incoming: Optional[dict], strict: bool, *, need_value: str = "a state dict") -> LoadReport:
        report = LoadReport()
        if incoming is None:
            report.problems.append(f"the loading rank was given no {need_value}")
            return report
        report.missing = [n for n in self.entries if n not in incoming]
        report.unexpected = [n for n in incoming if n not in self.entries]
        if strict and report.missing:
            report.problems.append(f"keys absent from the state dict: {report.missing}")
        if strict and report.unexpected:
            report.problems.append(f"keys the model does not have: {report.unexpected}")
        for name, entry in self.entries.items():
            if name not in incoming:
                continue
            report.present.append(name)
            if entry.full_shape is None:
                continue
            value = incoming[name]
            if not isinstance(value, torch.Tensor):
                report.problems.append(f"{name} should be a tensor, found {type(value).__name__}")
            elif tuple(value.shape) != tuple(entry.full_shape):
                report.problems.append(f"{name} has shape {tuple(value.shape)}, the model needs "
                                       f"{tuple(entry.full_shape)}")
        return report


def share_report(report: Optional[LoadReport], src: int, group=None) -> LoadReport:
    """Broadcast the loading rank's report (``src`` is a global rank)."""
    if not dist.is_initialized():
        return report
    box = [report]
    dist.broadcast_object_list(box, src=src, group=group)
    return box[0]


def parameter_names(module: nn.Module) -> dict[int, tuple[str, ...]]:
    """Every state-dict name of each parameter (tied weights have several),
    keyed by ``id(parameter)``; raises if a parameter has none."""
    names: dict[int, list[str]] = {id(p): [] for p in module.parameters()}
    for name, value in module.state_dict(keep_vars=True).items():
        if id(value) in names:
            names[id(value)].append(name)
    orphans = [n for n, p in module.named_parameters() if not names[id(p)]]
    if orphans:
        raise RuntimeError(f"parameters {orphans} do not appear in model.state_dict(); they could not be "
                           "checkpointed")
    return {k: tuple(v) for k, v in names.items()}


# --------------------------------------------------------------------------- TP shard transport
def tp_assemble(local: torch.Tensor, dim: Optional[int], group, tp_size: int, *, root_only: bool,
                i_am_root: bool) -> Optional[torch.Tensor]:
    """Join the TP shards of one tensor along ``dim``.  ``dim is None`` means
    the tensor is replicated and the local copy is the full one.  With
    ``root_only`` the shards are gathered to TP rank 0 (others get None);
    otherwise every rank joins (all-gather)."""
    if dim is None:
        return local.detach() if (i_am_root or not root_only) else None
    local = local.detach().contiguous()
    if root_only:
        parts = [torch.empty_like(local) for _ in range(tp_size)] if i_am_root else None
        dist.gather(local, gather_list=parts, dst=dist.get_global_rank(group, 0), group=group)
        return torch.cat(parts, dim=dim) if i_am_root else None
    parts = [torch.empty_like(local) for _ in range(tp_size)]
    dist.all_gather(parts, local, group=group)
    return torch.cat(parts, dim=dim)


def tp_distribute(full: Optional[torch.Tensor], dim: Optional[int], local_shape, dtype, device, group,
                  tp_size: int, i_am_root: bool) -> torch.Tensor:
    """Inverse of ``tp_assemble``: TP rank 0 holds ``full``; every rank returns
    its shard along ``dim`` (or the whole tensor when ``dim is None``) as a
    ``dtype`` tensor of ``local_shape`` on ``device``."""
    src = dist.get_global_rank(group, 0)
    out = torch.empty(tuple(local_shape), dtype=dtype, device=device)
    if dim is None:
        if i_am_root:
            out.copy_(full)
        dist.broadcast(out, src=src, group=group)
        return out
    pieces = ([p.contiguous() for p in full.to(device=device, dtype=dtype).chunk(tp_size, dim=dim)]
              if i_am_root else None)
    dist.scatter(out, scatter_list=pieces, src=src, group=group)
    return out
