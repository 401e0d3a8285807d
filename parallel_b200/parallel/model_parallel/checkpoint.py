"""Checkpoint adapters for model-parallel models.

* ``ModelParallelCheckpoint`` (TP/EP without FSDP): the portable state dict
  is gathered over TP along each parameter's ``shard_dim`` (and replicated
  parameters taken from TP rank 0); loading scatters / broadcasts.
  Exact-topology layout ``{"kind": "model-parallel", "plan", "state"}``.
* ``ComposedModelParallelCheckpoint`` (TP/EP over FSDP): FSDP's full local
  state, then TP gather to the portable root; loading goes portable -> TP
  scatter -> ``FSDPWrapper.load_local_full_state_dict``.  Layout
  ``{"kind": "model-parallel-fsdp", "plan", "fsdp"}``.

Formats and key order are the reference's (parallel/parallel/engine/
model_parallel/checkpoint.py) so checkpoints interchange.
"""
from __future__ import annotations

import copy
from collections import OrderedDict

import torch
import torch.distributed as dist
import torch.nn as nn

from ...state import Strategies
from .plan import ModelParallelPlan


def _cpu(t: torch.Tensor) -> torch.Tensor:
    return t.detach().to(device="cpu", copy=True)


def _mesh_rank(pconfig, dim: Strategies) -> int:
    mesh = pconfig.device_mesh
    if mesh is not None and dim.value in mesh.mesh_dim_names:
        return mesh.get_local_rank(dim.value)
    return 0


def _broadcast_validation(validation):
    if not dist.is_initialized():
        return validation
    payload = [validation if dist.get_rank() == 0 else None]
    dist.broadcast_object_list(payload, src=0)
    return payload[0]


class ModelParallelCheckpoint:
    def __init__(self, model, pconfig, plan: ModelParallelPlan, tp_mesh, device):
        self.model, self.pconfig, self.plan, self.tp_mesh = model, pconfig, plan, tp_mesh
        self.tp_group = tp_mesh.get_group()
        self.device = torch.device(device)
        ids = {id(p) for p in model.parameters()}
        self._parameter_names = {n for n, v in model.state_dict(keep_vars=True).items() if id(v) in ids}

    @property
    def is_active(self) -> bool:
        return True

    def _checkpoint_replica(self) -> bool:
        return _mesh_rank(self.pconfig, Strategies.DP_REPLICATE) == 0

    def _full_state_root(self) -> bool:
        return self._checkpoint_replica() and self.tp_mesh.get_local_rank() == 0

    def _gather(self, t: torch.Tensor, dim: int) -> torch.Tensor:
        parts = [torch.empty_like(t) for _ in range(self.tp_mesh.size())]
        dist.all_gather(parts, t.detach().contiguous(), group=self.tp_group)
        return torch.cat(parts, dim=dim)

    def full_state_dict(self):
        if not self._checkpoint_replica():
            return None
        local = self.model.state_dict(keep_vars=True)
        root = self._full_state_root()
        out = OrderedDict() if root else None
        seen: dict[int, torch.Tensor] = {}
        for name, v in local.items():
            if name in self._parameter_names:
                pl = self.plan.placement_for_parameter(name)
                full = (v.detach() if root else None) if pl.shard_dim is None else self._gather(v, pl.shard_dim)
                if root:
                    cpu = seen.get(id(v))
                    if cpu is None:
                        cpu = _cpu(full)
                        seen[id(v)] = cpu
                    out[name] = cpu
            elif root:
                out[name] = _cpu(v) if isinstance(v, torch.Tensor) else copy.deepcopy(v)
        if root and hasattr(local, "_metadata"):
            out._metadata = copy.deepcopy(local._metadata)
        return out

    def _validate(self, sd, strict: bool) -> dict:
        exp_state = self.model.state_dict()
        expected, actual = set(exp_state), set(sd) if sd is not None else set()
        missing, unexpected = sorted(expected - actual), sorted(actual - expected)
        errors = []
        if sd is None:
            errors.append("global rank zero requires a full state dict")
        if strict and missing:
            errors.append(f"Missing key(s): {missing}")
        if strict and unexpected:
            errors.append(f"Unexpected key(s): {unexpected}")
        if sd is not None:
            for n in expected & actual:
                src = sd[n]
                if not isinstance(src, torch.Tensor):
                    errors.append(f"Expected tensor for {n}")
                    continue
                shape = list(exp_state[n].shape)
                if n in self._parameter_names:
                    pl = self.plan.placement_for_parameter(n)
                    if pl.shard_dim is not None:
                        shape[pl.shard_dim] *= self.tp_mesh.size()
                if tuple(src.shape) != tuple(shape):
                    errors.append(f"Shape mismatch for {n}: expected {tuple(shape)}, got {tuple(src.shape)}")
        return {"error": "; ".join(errors) if errors else None, "missing": missing, "unexpected": unexpected,
                "available": sorted(actual & expected)}

    def _replica_root_tensor(self, source, shape, dtype):
        if self.tp_mesh.get_local_rank() != 0:
            return None
        t = source.to(self.device) if self._checkpoint_replica() else torch.empty(shape, dtype=dtype,
                                                                                   device=self.device)
        group = self.pconfig.group(Strategies.DP_REPLICATE)
        if group is not None and self.pconfig.dp_replicate_size > 1:
            dist.broadcast(t, src=dist.get_global_rank(group, 0), group=group)
        return t

    def load_full_state_dict(self, state_dict, strict: bool = True):
        root = not dist.is_initialized() or dist.get_rank() == 0
        validation = _broadcast_validation(self._validate(state_dict, strict) if root else None)
        if validation["error"]:
            raise RuntimeError(f"Error(s) in loading state_dict: {validation['error']}")
        dest_state = self.model.state_dict(keep_vars=True)
        tp_root = dist.get_global_rank(self.tp_group, 0)
        tp_rank = self.tp_mesh.get_local_rank()
        for name, dst in dest_state.items():
            if name not in validation["available"]:
                continue
            pl = self.plan.placement_for_parameter(name) if name in self._parameter_names else None
            local_shape = tuple(dst.shape)
            full_shape = list(local_shape)
            if pl is not None and pl.shard_dim is not None:
                full_shape[pl.shard_dim] *= self.tp_mesh.size()
            src = state_dict[name] if root and name in state_dict else None
            rep = self._replica_root_tensor(src, tuple(full_shape), dst.dtype)
            if pl is not None and pl.shard_dim is not None:
                recv = torch.empty_like(dst, device=self.device)
                lst = ([s.contiguous() for s in rep.chunk(self.tp_mesh.size(), dim=pl.shard_dim)]
                       if tp_rank == 0 else None)
                dist.scatter(recv, scatter_list=lst, src=tp_root, group=self.tp_group)
            else:
                recv = rep if tp_rank == 0 else torch.empty(local_shape, dtype=dst.dtype, device=self.device)
                dist.broadcast(recv, src=tp_root, group=self.tp_group)
            dst.detach().copy_(recv.to(dst.device))
        return nn.modules.module._IncompatibleKeys(validation["missing"], validation["unexpected"])

    def checkpoint_layout(self) -> dict:
        state = self.model.state_dict()
        return {
            "kind": "model-parallel",
            "plan": self.plan.checkpoint_metadata(),
            "state": [
                {"name": n, "local_shape": list(v.shape), "dtype": str(v.dtype),
                 "placement": (self.plan.placement_for_parameter(n).parallelism.value
                               if n in self._parameter_names else "buffer"),
                 "shard_dim": (self.plan.placement_for_parameter(n).shard_dim
                               if n in self._parameter_names else None)}
                for n, v in state.items()
            ],
        }

    def sharded_state_dict(self) -> dict:
        state = self.model.state_dict()
        return {"layout": self.checkpoint_layout(), "local_state": OrderedDict((n, _cpu(v)) for n, v in state.items())}

    def load_sharded_state_dict(self, state_dict, strict: bool = True):
        if not isinstance(state_dict, dict):
            raise TypeError("Sharded checkpoint state must be a dictionary")
        if state_dict.get("layout") != self.checkpoint_layout():
            raise RuntimeError("Sharded checkpoint layout does not match the current model")
        local = state_dict.get("local_state")
        if not isinstance(local, dict):
            raise TypeError("Sharded checkpoint has no local_state dictionary")
        return self.model.load_state_dict(local, strict=strict)


class ComposedModelParallelCheckpoint:
    def __init__(self, model, pconfig, plan, tp_mesh, fsdp_wrapper, device):
        self.model, self.pconfig, self.plan, self.tp_mesh = model, pconfig, plan, tp_mesh
        self.tp_group = tp_mesh.get_group()
        self.fsdp = fsdp_wrapper
        self.device = torch.device(device)
        self._local_shapes = {}
        for u in fsdp_wrapper.units:
            for m in u.param_metas:
                for n in fsdp_wrapper._parameter_state_names[id(m.parameter)]:
                    self._local_shapes[n] = tuple(m.shape)

    @property
    def _checkpoint_replica(self) -> bool:
        return _mesh_rank(self.pconfig, Strategies.DP_REPLICATE) == 0

    @property
    def _dp_shard_root(self) -> bool:
        return _mesh_rank(self.pconfig, Strategies.DP_SHARD) == 0

    @property
    def _portable_root(self) -> bool:
        return self._checkpoint_replica and self._dp_shard_root and self.tp_mesh.get_local_rank() == 0

    def _is_parameter(self, name: str) -> bool:
        return name in self.fsdp._parameter_state_keys

    def full_state_dict(self):
        local = self.fsdp.full_state_dict()
        if not self._checkpoint_replica or not self._dp_shard_root:
            return None
        root = self._portable_root
        out = OrderedDict() if root else None
        tp_root = dist.get_global_rank(self.tp_group, 0)
        for name in self.fsdp._state_dict_keys:
            v = local[name]
            pl = self.plan.placement_for_parameter(name) if self._is_parameter(name) else None
            if pl is not None and pl.shard_dim is not None:
                lv = v.to(self.device)
                parts = [torch.empty_like(lv) for _ in range(self.tp_mesh.size())] if root else None
                dist.gather(lv, gather_list=parts, dst=tp_root, group=self.tp_group)
                if root:
                    out[name] = _cpu(torch.cat(parts, dim=pl.shard_dim))
            elif root:
                out[name] = _cpu(v)
        if root and hasattr(local, "_metadata"):
            out._metadata = copy.deepcopy(local._metadata)
        return out

    def _validate(self, sd, strict: bool) -> dict:
        expected = set(self.fsdp._state_dict_keys)
        actual = set(sd) if sd is not None else set()
        missing, unexpected = sorted(expected - actual), sorted(actual - expected)
        errors = []
        if sd is None:
            errors.append("global rank zero requires a portable state dict")
        if strict and missing:
            errors.append(f"Missing key(s): {missing}")
        if strict and unexpected:
            errors.append(f"Unexpected key(s): {unexpected}")
        if sd is not None:
            cur = self.model.state_dict()
            for n in expected & actual:
                src = sd[n]
                if not isinstance(src, torch.Tensor):
                    errors.append(f"Expected tensor for {n}")
                    continue
                if self._is_parameter(n):
                    shape = list(self._local_shapes[n])
                    pl = self.plan.placement_for_parameter(n)
                    if pl.shard_dim is not None:
                        shape[pl.shard_dim] *= self.tp_mesh.size()
                else:
                    shape = list(cur[n].shape)
                if tuple(src.shape) != tuple(shape):
                    errors.append(f"Shape mismatch for {n}: expected {tuple(shape)}, got {tuple(src.shape)}")
        return {"error": "; ".join(errors) if errors else None, "missing": missing, "unexpected": unexpected,
                "available": sorted(expected & actual)}

    def _local_state_from_portable(self, sd, validation):
        if not self._checkpoint_replica or not self._dp_shard_root:
            return None
        root = self._portable_root
        tp_root = dist.get_global_rank(self.tp_group, 0)
        out = OrderedDict()
        cur = self.model.state_dict()
        for name in self.fsdp._state_dict_keys:
            if name not in validation["available"]:
                continue
            if self._is_parameter(name):
                pl = self.plan.placement_for_parameter(name)
                shape = self._local_shapes[name]
            else:
                pl, shape = None, tuple(cur[name].shape)
            src = sd[name].to(self.device) if root else None
            recv = torch.empty(shape, dtype=(sd[name].dtype if root else cur[name].dtype), device=self.device)
            if pl is not None and pl.shard_dim is not None:
                lst = [s.contiguous() for s in src.chunk(self.tp_mesh.size(), dim=pl.shard_dim)] if root else None
                dist.scatter(recv, scatter_list=lst, src=tp_root, group=self.tp_group)
            else:
                if root:
                    recv.copy_(src)
                dist.broadcast(recv, src=tp_root, group=self.tp_group)
            out[name] = _cpu(recv)
        return out

    def load_full_state_dict(self, state_dict, strict: bool = True):
        validation = _broadcast_validation(self._validate(state_dict, strict) if dist.get_rank() == 0 else None)
        if validation["error"] is not None:
            raise RuntimeError(f"Error(s) in loading portable state_dict: {validation['error']}")
        local = self._local_state_from_portable(state_dict, validation)
        self.fsdp.load_local_full_state_dict(local, strict=strict)
        return nn.modules.module._IncompatibleKeys(validation["missing"], validation["unexpected"])

    def checkpoint_layout(self) -> dict:
        return {"kind": "model-parallel-fsdp", "plan": self.plan.checkpoint_metadata(),
                "fsdp": self.fsdp.checkpoint_layout()}

    def sharded_state_dict(self) -> dict:
        return {"layout": self.checkpoint_layout(), "fsdp": self.fsdp.sharded_state_dict()}

    def load_sharded_state_dict(self, state_dict, strict: bool = True):
        if not isinstance(state_dict, dict):
            raise TypeError("Sharded checkpoint state must be a dictionary")
        if state_dict.get("layout") != self.checkpoint_layout():
            raise RuntimeError("Composite checkpoint layout does not match the model")
        return self.fsdp.load_sharded_state_dict(state_dict["fsdp"], strict=strict)
