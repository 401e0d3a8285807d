"""State dicts of an FSDP-wrapped model (mixed into ``FSDPWrapper``).

What has to match the reference (``parallel/parallel/engine/dp_sharded.py:
540-868``) is the data, not the code: the portable dict is the plain
``model.state_dict()`` with full tensors; the exact-topology payload is
``{"layout", "shards", "non_parameter_state"}`` (``{"layout",
"full_state"}`` when FSDP is inactive) with ``checkpoint_layout()`` as the
layout dict.  How it is produced here:

* a unit is the transport: saving gathers one unit at a time into its full
  buffer and copies the parameters out on the dp_shard root; loading fills
  the root's full buffer, broadcasts the whole buffer over the shard group in
  one collective and writes every rank's rows back (``writeback_shards``);
* validation is ``state_io.StateCatalog.audit`` against ``local_catalog()``
  (full parameter shapes from the unit metas), computed by the loading rank
  and broadcast, so every rank raises together;
* after a load, replica 0 of the dp_replicate dimension broadcasts shards
  and buffers to the other replicas.
"""
from __future__ import annotations

from collections import OrderedDict
from contextlib import contextmanager
from typing import Any, Optional

import torch
import torch.distributed as dist

from ..state import Strategies
from .fsdp_utils import local_tensor
from .state_io import (Entry, LoadReport, StateCatalog, host_tensor, parameter_names, share_report,
                       with_metadata)


class FSDPStateMixin:
    """Needs ``model``, ``pconfig``, ``units``, ``dp_shard_group``, ``device``,
    ``is_active`` and ``get_sharded_params`` from the wrapper."""

    # ------------------------------------------------------------------ naming
    def _index_state(self) -> None:
        """Record the model's state-dict keys and each parameter's names (a
        tied weight has several); the wrapper shares one tensor between them."""
        self.state_names: dict[int, tuple[str, ...]] = parameter_names(self.model)
        self.state_keys: tuple[str, ...] = tuple(self.model.state_dict(keep_vars=True).keys())
        self.param_keys: set[str] = {n for names in self.state_names.values() for n in names}

    def _ensure_indexed(self) -> None:
        if not getattr(self, "state_keys", None):
            self._index_state()

    def local_catalog(self) -> StateCatalog:
        """Entries of the (model-parallel-local) full state dict, with the full
        parameter shapes the units reassemble."""
        self._ensure_indexed()
        full_shapes = {}
        for unit in self.units:
            for meta in unit.param_metas:
                for name in self.state_names[id(meta.parameter)]:
                    full_shapes[name] = (tuple(meta.shape), meta.parameter.dtype)
        entries = []
        for name, value in self.model.state_dict(keep_vars=True).items():
            if name in full_shapes:
                shape, dtype = full_shapes[name]
            elif isinstance(value, torch.Tensor):
                shape, dtype = tuple(value.shape), value.dtype
            else:
                shape, dtype = None, None
            entries.append(Entry(name, name in self.param_keys, shape, dtype))
        return StateCatalog(entries)

    # ------------------------------------------------------------------ rank roles
    def _coordinate(self, dim: Strategies) -> int:
        mesh = self.pconfig.device_mesh
        names = tuple(getattr(mesh, "mesh_dim_names", None) or ()) if mesh is not None else ()
        return mesh.get_local_rank(dim.value) if dim.value in names else 0

    def _replica_zero(self) -> bool:
        return self._coordinate(Strategies.DP_REPLICATE) == 0

    def _holds_full_state(self) -> bool:
        """The rank that assembles / consumes the full dict of its replica."""
        if not self._replica_zero():
            return False
        if self.is_active:
            return dist.get_rank(self.dp_shard_group) == 0
        return not dist.is_initialized() or dist.get_rank() == 0

    @contextmanager
    def _unit_gathered(self, unit):
        """The unit's full parameters for the duration of the block (left as
        they were found afterwards)."""
        already = unit.gathered
        unit.all_gather()
        try:
            yield unit
        finally:
            if not already:
                unit.free_full_params()

    # ------------------------------------------------------------------ transport helpers
    def _broadcast_in(self, tensor: torch.Tensor, group) -> None:
        """Broadcast ``tensor`` from the group's first rank, staging through the
        device when it lives elsewhere (host shards under CPU offload)."""
        value = local_tensor(tensor).detach()
        src = dist.get_global_rank(group, 0)
        if value.device.type == self.device.type:
            dist.broadcast(value, src=src, group=group)
        else:
            staged = value.to(self.device)
            dist.broadcast(staged, src=src, group=group)
            value.copy_(staged.to(value.device))

    def _replicas_follow_zero(self) -> None:
        """After a load: replica 0's shards and buffers to every replica."""
        group = self.pconfig.group(Strategies.DP_REPLICATE)
        if group is None:
            return
        params = self.get_sharded_params() if self.is_active else list(self.model.parameters())
        for tensor in list(self.model.buffers()) + params:
            self._broadcast_in(tensor, group)

    def _non_parameter_state(self) -> OrderedDict:
        current = self.model.state_dict(keep_vars=True)
        out = OrderedDict((n, host_tensor(v)) for n, v in current.items() if n not in self.param_keys)
        return with_metadata(out, current)

    def _assign_non_parameter_state(self, incoming) -> None:
        for name, dst in self.model.state_dict(keep_vars=True).items():
            if name not in self.param_keys and name in incoming and isinstance(dst, torch.Tensor):
                dst.detach().copy_(incoming[name])

    # ------------------------------------------------------------------ portable dict
    def full_state_dict(self) -> Optional[OrderedDict]:
        """Full CPU state dict on the replica-0 dp_shard root, else None
        (collective over the shard group)."""
        self._ensure_indexed()
        if not self._replica_zero():
            return None
        holder = self._holds_full_state()
        if not self.is_active:
            if not holder:
                return None
            current = self.model.state_dict(keep_vars=True)
            return with_metadata(OrderedDict((n, host_tensor(v)) for n, v in current.items()), current)
        copies: dict[str, torch.Tensor] = {}
        for unit in self.units:
            with self._unit_gathered(unit):
                if holder:
                    for meta in unit.param_metas:
                        tensor = host_tensor(meta.parameter)
                        copies.update((n, tensor) for n in self.state_names[id(meta.parameter)])
        if not holder:
            return None
        rest = self._non_parameter_state()
        return with_metadata(OrderedDict((n, copies[n] if n in copies else rest[n]) for n in self.state_keys), rest)

    def _restore_full(self, incoming, holder: bool, strict: bool) -> None:
        """Fill the model from ``incoming`` (held by ``holder``, the shard
        group's first rank) on the ranks of replica 0."""
        if not self.is_active:
            if holder:
                self.model.load_state_dict(incoming, strict=strict)
            return
        root = dist.get_global_rank(self.dp_shard_group, 0)
        for unit in self.units:
            with self._unit_gathered(unit):
                if holder:
                    for meta in unit.param_metas:
                        name = next((n for n in self.state_names[id(meta.parameter)] if n in incoming), None)
                        if name is not None:
                            meta.parameter.detach().copy_(incoming[name])
                dist.broadcast(unit.full_buffer, src=root, group=self.dp_shard_group)
                unit.writeback_shards()
        if holder:
            self._assign_non_parameter_state(incoming)
        for buf in self.model.buffers():
            self._broadcast_in(buf, self.dp_shard_group)

    def load_full_state_dict(self, state_dict, strict: bool = True):
        """Load a portable dict given on global rank 0 (collective)."""
        self._ensure_indexed()
        loader = not dist.is_initialized() or dist.get_rank() == 0
        report = self.local_catalog().audit(state_dict, strict) if loader else None
        report = share_report(report, src=0)
        report.raise_if_bad("the state dict")
        if self._replica_zero():
            self._restore_full(state_dict, self._holds_full_state(), strict)
        self._replicas_follow_zero()
        return report.incompatible_keys()

    def load_local_full_state_dict(self, state_dict, strict: bool = True):
        """Load a model-parallel-local full dict given on each replica-0
        dp_shard root (the composed model-parallel checkpoint's path)."""
        if not self.is_active:
            return self.load_full_state_dict(state_dict, strict=strict)
        self._ensure_indexed()
        report = LoadReport()
        if self._replica_zero():
            holder = dist.get_rank(self.dp_shard_group) == 0
            report = self.local_catalog().audit(state_dict, strict, need_value="local state dict") if holder else None
            report = share_report(report, src=dist.get_global_rank(self.dp_shard_group, 0), group=self.dp_shard_group)
            report.raise_if_bad("the model-parallel-local state dict")
            self._restore_full(state_dict, holder, strict)
        self._replicas_follow_zero()
        return report.incompatible_keys()

    def state_dict(self):
        return self.full_state_dict()

    def load_state_dict(self, state_dict, strict: bool = True):
        return self.load_full_state_dict(state_dict, strict=strict)

    # ------------------------------------------------------------------ exact-topology payload
    def checkpoint_layout(self) -> dict[str, Any]:
        """The unit / parameter description stored in the manifest (an
        interface: both implementations compare it for equality)."""
        self._ensure_indexed()

        def describe(meta):
            shard = meta.sharded_param
            return {"names": list(self.state_names[id(meta.parameter)]), "shape": list(meta.shape),
                    "stride": list(meta.stride), "numel": meta.numel,
                    "local_shape": list(shard._local_tensor.shape),
                    "placements": [str(p) for p in shard.placements],
                    "dtype": str(meta.parameter.dtype), "requires_grad": meta.parameter.requires_grad}

        return {"state_dict_keys": list(self.state_keys),
                "units": [{"unit_index": u.unit_index, "parameters": [describe(m) for m in u.param_metas]}
                          for u in self.units]}

    def sharded_state_dict(self) -> dict[str, Any]:
        self._ensure_indexed()
        if not self.is_active:
            return {"layout": self.checkpoint_layout(), "full_state": self.full_state_dict()}
        return {"layout": self.checkpoint_layout(), "shards": [host_tensor(p) for p in self.get_sharded_params()],
                "non_parameter_state": self._non_parameter_state()}

    def load_sharded_state_dict(self, state_dict, strict: bool = True):
        self._ensure_indexed()
        if not isinstance(state_dict, dict):
            raise TypeError(f"an FSDP shard payload is a dict, got {type(state_dict).__name__}")
        if state_dict.get("layout") != self.checkpoint_layout():
            raise RuntimeError("sharded checkpoint layout does not match the current model")
        if not self.is_active:
            return self.model.load_state_dict(state_dict["full_state"], strict=strict)
        params = self.get_sharded_params()
        shards = state_dict.get("shards", [])
        problems = []
        if len(shards) != len(params):
            problems.append(f"checkpoint holds {len(shards)} parameter shards, this model has {len(params)}")
        for i, (param, shard) in enumerate(zip(params, shards)):
            want = param._local_tensor
            if not isinstance(shard, torch.Tensor) or shard.shape != want.shape or shard.dtype != want.dtype:
                got = (tuple(shard.shape), shard.dtype) if isinstance(shard, torch.Tensor) else type(shard).__name__
                problems.append(f"parameter shard {i} is {got}, expected {(tuple(want.shape), want.dtype)}")
        rest = state_dict.get("non_parameter_state", {})
        if not isinstance(rest, dict):
            raise TypeError("non_parameter_state of an FSDP shard payload must be a dict")
        wanted = OrderedDict((n, v) for n, v in self.model.state_dict(keep_vars=True).items()
                             if n not in self.param_keys)
        missing = [n for n in wanted if n not in rest]
        unexpected = [n for n in rest if n not in wanted]
        if strict and missing:
            problems.append(f"non-parameter keys absent from the checkpoint: {missing}")
        if strict and unexpected:
            problems.append(f"non-parameter keys the model does not have: {unexpected}")
        for name, dst in wanted.items():
            if name in rest and isinstance(dst, torch.Tensor):
                src = rest[name]
                if not isinstance(src, torch.Tensor) or src.shape != dst.shape or src.dtype != dst.dtype:
                    problems.append(f"non-parameter state {name} does not match the model's shape / dtype")
        if problems:
            raise RuntimeError("; ".join(problems))
        for param, shard in zip(params, shards):
            param._local_tensor.detach().copy_(shard)
        self._assign_non_parameter_state(rest)
        return LoadReport(missing, unexpected).incompatible_keys()
