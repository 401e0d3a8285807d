"""Checkpoint adapters for model-parallel models.

A model-parallel rank holds TP / EP shards of the parameters.  The portable
state dict is the HF-layout full model; converting between the two is a join
(or split) of every parameter along its plan ``shard_dim`` over the TP group,
with replicated parameters and buffers taken from TP rank 0.  Two adapters
differ only in where the rank-local tensors live:

* ``ModelParallelCheckpoint`` (TP / EP without FSDP): in the module itself.
  Exact-topology layout ``{"kind": "model-parallel", "plan", "state"}``; the
  sharded payload is ``{"layout", "local_state"}``.
* ``ComposedModelParallelCheckpoint`` (TP / EP over FSDP): in the FSDP
  units, whose ``full_state_dict`` / ``load_local_full_state_dict`` produce
  and accept the model-parallel-local full state on the dp_shard root.
  Layout ``{"kind": "model-parallel-fsdp", "plan", "fsdp"}``; the sharded
  payload is ``{"layout", "fsdp"}``.

Both validate an incoming portable dict with the shared
``state_io.StateCatalog`` (full shapes = local shapes with the shard
dimension multiplied by the TP size) on global rank 0 and share the verdict
with every rank before any tensor moves.  Formats and key order are the
reference's (``parallel/parallel/engine/model_parallel/checkpoint.py``), so
checkpoints interchange.
"""
from __future__ import annotations

from collections import OrderedDict
from typing import Optional

import torch
import torch.distributed as dist

from ...state import Strategies
from ..state_io import (Entry, LoadReport, StateCatalog, host_tensor, parameter_names, share_report, tp_assemble,
                        tp_distribute, with_metadata)
from .plan import ModelParallelPlan


def _coordinate(pconfig, dim: Strategies) -> int:
    mesh = pconfig.device_mesh
    names = tuple(getattr(mesh, "mesh_dim_names", None) or ()) if mesh is not None else ()
    return mesh.get_local_rank(dim.value) if dim.value in names else 0


class _TPStateAdapter:
    """Shared machinery: the catalog, the TP join / split loops and the
    replica fan-out; subclasses say where local tensors come from / go to."""

    def __init__(self, model, pconfig, plan: ModelParallelPlan, tp_mesh, device):
        self.model, self.pconfig, self.plan, self.tp_mesh = model, pconfig, plan, tp_mesh
        self.tp_group = tp_mesh.get_group()
        self.tp_size = tp_mesh.size()
        self.device = torch.device(device)

    # -------------------------------------------------------------- rank roles
    @property
    def tp_rank(self) -> int:
        return self.tp_mesh.get_local_rank()

    @property
    def replica_zero(self) -> bool:
        return _coordinate(self.pconfig, Strategies.DP_REPLICATE) == 0

    def split_dim(self, name: str) -> Optional[int]:
        return self.plan.placement_for_parameter(name).shard_dim

    def _entry(self, name: str, local_shape, dtype, is_param: bool) -> Entry:
        dim = self.split_dim(name) if is_param else None
        full = list(local_shape)
        if dim is not None:
            full[dim] *= self.tp_size
        return Entry(name, is_param, tuple(full), dtype, dim)

    # -------------------------------------------------------------- subclass interface
    def catalog(self) -> StateCatalog:
        raise NotImplementedError

    # -------------------------------------------------------------- portable save
    def _join(self, local_state, *, dedupe: bool) -> Optional[OrderedDict]:
        """Portable state on TP rank 0 (None elsewhere) from this rank's local
        tensors; every TP rank of the group must call."""
        root = self.tp_rank == 0
        out = OrderedDict() if root else None
        # id -> portable tensor (None off the root); every rank records it so
        # all ranks skip the same collectives for a tied weight's second name
        joined: dict[int, Optional[torch.Tensor]] = {}
        for entry in self.catalog():
            value = local_state[entry.name]
            if not entry.is_param:
                if root:
                    out[entry.name] = host_tensor(value)
                continue
            if dedupe and id(value) in joined:  # tied weights stay one tensor
                if root:
                    out[entry.name] = joined[id(value)]
                continue
            full = tp_assemble(value.to(self.device), entry.tp_dim, self.tp_group, self.tp_size,
                               root_only=True, i_am_root=root)
            joined[id(value)] = host_tensor(full) if root else None
            if root:
                out[entry.name] = joined[id(value)]
        return out

    # -------------------------------------------------------------- portable load
    def _verdict(self, state_dict, strict: bool) -> LoadReport:
        loader = not dist.is_initialized() or dist.get_rank() == 0
        report = self.catalog().audit(state_dict, strict, need_value="portable state dict") if loader else None
        report = share_report(report, src=0)
        report.raise_if_bad("the portable state dict")
        return report

    def _split(self, state_dict, report: LoadReport, local_shapes: dict, dtypes: dict):
        """Yield (name, local tensor) for each present entry; TP rank 0 of the
        participating group holds ``state_dict`` (the portable dict)."""
        root = self.tp_rank == 0
        for entry in self.catalog():
            if entry.name not in report.present:
                continue
            full = state_dict[entry.name] if root else None
            yield entry.name, tp_distribute(full, entry.tp_dim, local_shapes[entry.name], dtypes[entry.name],
                                            self.device, self.tp_group, self.tp_size, root)


class ModelParallelCheckpoint(_TPStateAdapter):
    """TP / EP shards held by the module itself (no FSDP)."""

    def __init__(self, model, pconfig, plan: ModelParallelPlan, tp_mesh, device):
        super().__init__(model, pconfig, plan, tp_mesh, device)
        self._param_keys = {n for names in parameter_names(model).values() for n in names}

    @property
    def is_active(self) -> bool:
        return True

    def catalog(self) -> StateCatalog:
        return StateCatalog(self._entry(n, v.shape, v.dtype, n in self._param_keys)
                            for n, v in self.model.state_dict(keep_vars=True).items())

    def full_state_dict(self):
        if not self.replica_zero:
            return None
        local = self.model.state_dict(keep_vars=True)
        out = self._join(local, dedupe=True)
        return with_metadata(out, local) if out is not None else None

    def _from_replica_zero(self, tensor: Optional[torch.Tensor], shape, dtype) -> Optional[torch.Tensor]:
        """TP rank 0 of every replica gets replica 0's full tensor."""
        if self.tp_rank != 0:
            return None
        if self.replica_zero:
            tensor = tensor.to(self.device)
        else:
            tensor = torch.empty(shape, dtype=dtype, device=self.device)
        group = self.pconfig.group(Strategies.DP_REPLICATE)
        if group is not None and self.pconfig.dp_replicate_size > 1:
            dist.broadcast(tensor, src=dist.get_global_rank(group, 0), group=group)
        return tensor

    def load_full_state_dict(self, state_dict, strict: bool = True):
        report = self._verdict(state_dict, strict)
        catalog = self.catalog()
        dest = self.model.state_dict(keep_vars=True)
        # replica fan-out first, then the TP split of each tensor
        staged = {}
        for name in report.present:
            src = state_dict[name] if (self.replica_zero and self.tp_rank == 0) else None
            staged[name] = self._from_replica_zero(src, catalog[name].full_shape, dest[name].dtype)
        shapes = {n: tuple(dest[n].shape) for n in report.present}
        dtypes = {n: dest[n].dtype for n in report.present}
        for name, local in self._split(staged, report, shapes, dtypes):
            dest[name].detach().copy_(local.to(dest[name].device))
        return report.incompatible_keys()

    def checkpoint_layout(self) -> dict:
        rows = []
        state = self.model.state_dict()
        for e in self.catalog():
            placement = self.plan.placement_for_parameter(e.name) if e.is_param else None
            rows.append({"name": e.name, "local_shape": list(state[e.name].shape), "dtype": str(e.dtype),
                         "placement": placement.parallelism.value if placement else "buffer",
                         "shard_dim": placement.shard_dim if placement else None})
        return {"kind": "model-parallel", "plan": self.plan.checkpoint_metadata(), "state": rows}

    def sharded_state_dict(self) -> dict:
        return {"layout": self.checkpoint_layout(),
                "local_state": OrderedDict((n, host_tensor(v)) for n, v in self.model.state_dict().items())}

    def load_sharded_state_dict(self, state_dict, strict: bool = True):
        if not isinstance(state_dict, dict) or not isinstance(state_dict.get("local_state"), dict):
            raise TypeError("a model-parallel shard payload is a dict with a 'local_state' dict")
        if state_dict.get("layout") != self.checkpoint_layout():
            raise RuntimeError("sharded checkpoint layout does not match the current model")
        return self.model.load_state_dict(state_dict["local_state"], strict=strict)


class ComposedModelParallelCheckpoint(_TPStateAdapter):
    """TP / EP shards further row-sharded by FSDP units."""

    def __init__(self, model, pconfig, plan, tp_mesh, fsdp_wrapper, device):
        super().__init__(model, pconfig, plan, tp_mesh, device)
        self.fsdp = fsdp_wrapper

    @property
    def dp_shard_root(self) -> bool:
        return _coordinate(self.pconfig, Strategies.DP_SHARD) == 0

    def catalog(self) -> StateCatalog:
        local = self.fsdp.local_catalog()  # model-parallel-local full shapes
        return StateCatalog(self._entry(e.name, e.full_shape, e.dtype, e.is_param) for e in local)

    def full_state_dict(self):
        local = self.fsdp.full_state_dict()  # on every dp_shard root of replica 0
        if not (self.replica_zero and self.dp_shard_root):
            return None
        out = self._join(local, dedupe=False)
        return with_metadata(out, local) if out is not None else None

    def load_full_state_dict(self, state_dict, strict: bool = True):
        report = self._verdict(state_dict, strict)
        local = None
        if self.replica_zero and self.dp_shard_root:
            local_catalog = self.fsdp.local_catalog()
            shapes = {e.name: e.full_shape for e in local_catalog}
            dtypes = {e.name: e.dtype for e in local_catalog}
            local = OrderedDict((n, host_tensor(t)) for n, t in self._split(state_dict, report, shapes, dtypes))
        self.fsdp.load_local_full_state_dict(local, strict=strict)
        return report.incompatible_keys()

    def checkpoint_layout(self) -> dict:
        return {"kind": "model-parallel-fsdp", "plan": self.plan.checkpoint_metadata(),
                "fsdp": self.fsdp.checkpoint_layout()}

    def sharded_state_dict(self) -> dict:
        return {"layout": self.checkpoint_layout(), "fsdp": self.fsdp.sharded_state_dict()}

    def load_sharded_state_dict(self, state_dict, strict: bool = True):
        if not isinstance(state_dict, dict) or "fsdp" not in state_dict:
            raise TypeError("a composed shard payload is a dict with an 'fsdp' entry")
        if state_dict.get("layout") != self.checkpoint_layout():
            raise RuntimeError("composed checkpoint layout does not match the model")
        return self.fsdp.load_sharded_state_dict(state_dict["fsdp"], strict=strict)
