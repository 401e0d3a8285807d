"""One FSDP unit: a flat bucket of dim-0 parameter shards plus its collectives.

Layout (identical to the reference, parallel/parallel/engine/_dp_param_unit.py:
170-277, so sharded checkpoints interchange):
* every parameter is split by rows into ``padded_rows = ceil(rows / N)``-row
  shards; rank r owns rows [r*padded_rows, ...);
* the rank's *local bucket* concatenates its padded shards in parameter order;
* each sharded parameter is exposed as ``DTensor(Shard(0))`` over the local
  (unpadded) rows, which is what the optimizer and checkpoints see.

B200-specific differences:
* the gathered (full) parameters are written **parameter-major** - each
  parameter's N shards back to back, i.e. the full padded parameter - so
  adjacent parameters (q/k/v, gate/up) form one matrix for the fused GEMMs and
  no per-parameter unpack copies run on the P2P path;
* reduce-scatter inputs are packed straight from the gradients the unit's
  backward produced (no ``param.grad`` round trip).
"""
from __future__ import annotations

from dataclasses import dataclass, field
from typing import Optional

import torch
import torch.distributed as dist
import torch.nn as nn
from torch.distributed.tensor import DTensor, Shard


@dataclass
class ParamMeta:
    name: str
    shape: torch.Size
    stride: tuple
    numel: int
    parameter: nn.Parameter
    module_refs: list = field(default_factory=list)
    sharded_param: Optional[nn.Parameter] = None
    local_rows: int = 0
    padded_rows: int = 0
    bucket_offset: int = 0   # offset of this param's shard inside the local bucket
    padded_numel: int = 0    # numel of one padded shard
    full_offset: int = 0     # offset of the full padded param inside the gathered buffer
    row_numel: int = 1
    padded_shard: Optional[torch.Tensor] = None


class DPParamUnit:
    """Flat-bucket FSDP unit (see module docstring)."""

    def __init__(self, module: nn.Module, dp_shard_mesh, unit_index: int, collectives, *,
                 cpu_offload: bool = False, use_activation_checkpoint: bool = False, device=None,
                 named_parameters=None, reshard_after_forward: bool = True,
                 overlap_backward_reductions: bool = True):
        self.module = module
        self.mesh = dp_shard_mesh
        self.group = dp_shard_mesh.get_group()
        self.unit_index = unit_index
        self.coll = collectives
        self.cpu_offload = cpu_offload
        self.use_activation_checkpoint = use_activation_checkpoint
        self.reshard_after_forward = reshard_after_forward
        self.gradient_reduction_mode = "overlapped" if overlap_backward_reductions else "deferred"
        self._named_params = list(named_parameters if named_parameters is not None else module.named_parameters())
        if not self._named_params:
            raise ValueError(f"FSDP unit {unit_index}: no parameters to shard")
        rg = {p.requires_grad for _, p in self._named_params}
        if len(rg) != 1:
            raise ValueError(f"FSDP unit {unit_index}: trainable and frozen parameters must go to separate units")
        self.requires_grad = rg.pop()
        self.device = device or self._named_params[0][1].device
        self.world_size = self.mesh.size()
        self.rank = self.mesh.get_local_rank()
        self.param_metas: list[ParamMeta] = []
        self.bucket_numel = 0
        self.full_numel = 0
        self.local_bucket: Optional[torch.Tensor] = None     # [bucket_numel] params (persistent)
        self.grad_bucket: Optional[torch.Tensor] = None      # [bucket_numel] reduced grads (persistent)
        self.full_buffer: Optional[torch.Tensor] = None      # [full_numel] gathered params (transient)
        self.next_fwd: Optional["DPParamUnit"] = None
        self.next_bwd: Optional["DPParamUnit"] = None
        self._is_sharded = False
        self._gather_event = None
        self._pending = None        # in-flight reduce-scatter handle
        self._grad_valid = False    # grad_bucket holds a gradient for the current accumulation
        self._participation: Optional[list[bool]] = None
        self._prefetch_stream = torch.cuda.Stream(device=self.device) if self.device.type == "cuda" else None

    # ------------------------------------------------------------ sharding
    @property
    def parameters(self) -> list[nn.Parameter]:
        return [m.parameter for m in self.param_metas]

    @property
    def parameter_ids(self) -> set[int]:
        return {id(p) for _, p in self._named_params}

    def _find_module_refs(self, parameter):
        refs = []
        for module in self.module.modules():
            for name, cand in module._parameters.items():
                if cand is parameter:
                    refs.append((module, name))
        return refs

    def shard(self) -> None:
        if self._is_sharded:
            raise RuntimeError(f"FSDP unit {self.unit_index}: shard() was already called")
        N, r = self.world_size, self.rank
        self.param_metas.clear()
        for name, p in self._named_params:
            if isinstance(p, DTensor):
                raise NotImplementedError(f"FSDP unit {self.unit_index}: {name} is a DTensor; units shard plain local tensors")
            if p.ndim == 0:
                raise ValueError(f"FSDP unit {self.unit_index}: {name} is a scalar; dim-0 sharding needs rows")
            refs = self._find_module_refs(p)
            if not refs:
                raise RuntimeError(f"FSDP unit {self.unit_index}: {name} is not registered on any module of the unit")
            meta = ParamMeta(name=name, shape=p.shape, stride=tuple(p.stride()), numel=p.numel(), parameter=p,
                             module_refs=refs)
            meta.padded_rows = (p.shape[0] + N - 1) // N
            start = min(r * meta.padded_rows, p.shape[0])
            meta.local_rows = min(meta.padded_rows, p.shape[0] - start)
            meta.row_numel = p.numel() // p.shape[0] if p.shape[0] else 0
            self.param_metas.append(meta)
        off = foff = 0
        for m in self.param_metas:
            m.padded_numel = m.padded_rows * m.row_numel
            m.bucket_offset = off
            m.full_offset = foff
            off += m.padded_numel
            foff += m.padded_numel * N
        # 16-byte-align every full param start for TMA (bf16: multiples of 8)
        self.bucket_numel = off
        self.full_numel = foff
        dtype = self.param_metas[0].parameter.dtype
        if self.cpu_offload:
            # shards (and, via the optimizer, its state) live in pinned host memory;
            # the all-gather copies them to the device (the reference's cpu_offload,
            # parallel/parallel/engine/_dp_param_unit.py:205-214,518-533)
            self.local_bucket = torch.zeros(self.bucket_numel, dtype=dtype,
                                            pin_memory=torch.cuda.is_available() and self.device.type == "cuda")
        else:
            self.local_bucket = self.coll.alloc_local_bucket(self, self.bucket_numel, dtype, self.device)
        self.local_bucket.zero_()
        root = dist.get_global_rank(self.group, 0)
        for m in self.param_metas:
            full = m.parameter.detach().to(self.device).contiguous()
            dist.broadcast(full, src=root, group=self.group)
            shard = self.local_bucket.narrow(0, m.bucket_offset, m.padded_numel).view(m.padded_rows,
                                                                                   *m.shape[1:])
            start = min(r * m.padded_rows, m.shape[0])
            if m.local_rows:
                shard[: m.local_rows].copy_(full.narrow(0, start, m.local_rows))
            m.padded_shard = shard
            local = shard.narrow(0, 0, m.local_rows)
            dt = DTensor.from_local(local, device_mesh=self.mesh, placements=(Shard(0),), run_check=False,
                                    shape=m.shape, stride=m.stride)
            m.sharded_param = nn.Parameter(dt, requires_grad=m.parameter.requires_grad)
            self._set_registered(m, m.sharded_param)
            m.parameter.data = torch.empty(0, dtype=m.parameter.dtype, device=self.device)
        self._is_sharded = True

    def _set_registered(self, meta: ParamMeta, value) -> None:
        for module, name in meta.module_refs:
            module._parameters[name] = value

    def sharded_params(self) -> list[nn.Parameter]:
        return [m.sharded_param for m in self.param_metas]

    # ------------------------------------------------------------ gather / free
    @property
    def gathered(self) -> bool:
        return self.full_buffer is not None

    def _install_full(self, full: torch.Tensor) -> None:
        self.full_buffer = full
        for m in self.param_metas:
            rows = m.padded_rows * self.world_size
            view = full.narrow(0, m.full_offset, rows * m.row_numel).view(rows, *m.shape[1:])
            m.parameter.data = view.narrow(0, 0, m.shape[0])
            self._set_registered(m, m.parameter)

    def all_gather(self, *, mode: str = "demand") -> None:
        """Gather on the current stream (no-op if already gathered)."""
        if self.full_buffer is not None:
            self.wait_for_prefetch()
            return
        full = self.coll.all_gather(self, mode=mode)
        self._install_full(full)

    def prefetch(self) -> None:
        """Gather on the side stream; consumers call ``wait_for_prefetch``."""
        if self.full_buffer is not None:
            return
        if self._prefetch_stream is None:
            self.all_gather(mode="prefetch")
            return
        cur = torch.cuda.current_stream(self.device)
        self._prefetch_stream.wait_stream(cur)
        with torch.cuda.stream(self._prefetch_stream):
            full = self.coll.all_gather(self, mode="prefetch")
            ev = torch.cuda.Event()
            ev.record(self._prefetch_stream)
        self._install_full(full)
        self._gather_event = ev

    def wait_for_prefetch(self) -> None:
        if self._gather_event is not None:
            cur = torch.cuda.current_stream(self.device)
            cur.wait_event(self._gather_event)
            if self.full_buffer is not None:
                self.full_buffer.record_stream(cur)
            self._gather_event = None

    def free_full_params(self) -> None:
        if self.full_buffer is None:
            return
        self.wait_for_prefetch()
        for m in self.param_metas:
            self._set_registered(m, m.sharded_param)
            m.parameter.data = torch.empty(0, dtype=m.parameter.dtype, device=self.device)
        self.coll.release_full(self, self.full_buffer)
        self.full_buffer = None

    def writeback_shards(self) -> None:
        """Copy the gathered parameters into this rank's shards (checkpoint load)."""
        if self.full_buffer is None:
            raise RuntimeError(f"FSDP unit {self.unit_index}: write-back of shards needs the gathered parameters")
        for m in self.param_metas:
            start = min(self.rank * m.padded_rows, m.shape[0])
            m.padded_shard.zero_()
            if m.local_rows:
                m.padded_shard[: m.local_rows].copy_(m.parameter.detach().narrow(0, start, m.local_rows))

    # ------------------------------------------------------------ gradients
    def reduce_gradients(self, grads: list[Optional[torch.Tensor]]) -> None:
        """Launch the reduce-scatter of this unit's full gradients (async).

        ``grads[i]`` is the full gradient of ``param_metas[i]`` (None = no
        local gradient: zeros are contributed).  The result is averaged over
        the shard group and accumulated into ``grad_bucket``.
        """
        if self._pending is not None:
            raise RuntimeError(f"FSDP unit {self.unit_index}: its previous gradient reduction has not finished")
        self._participation = [g is not None for g in grads]
        accumulate = self._grad_valid
        if self.grad_bucket is None:
            self.grad_bucket = torch.zeros(self.bucket_numel, dtype=self.local_bucket.dtype, device=self.device)
        self._pending = self.coll.reduce_scatter(self, grads, self.grad_bucket, accumulate,
                                                 mode=self.gradient_reduction_mode)
        self._grad_valid = True

    def finish_gradient_reduction(self) -> None:
        if self._pending is None:
            return
        self.coll.wait(self._pending)
        self._pending = None

    @property
    def reduction_in_flight(self) -> bool:
        return self._pending is not None

    def attach_gradients(self, participation: Optional[list[bool]] = None) -> None:
        """Expose the reduced shard gradients as DTensor ``.grad`` views."""
        self.finish_gradient_reduction()
        if not self._grad_valid:
            return
        part = participation or [True] * len(self.param_metas)
        bucket = self.grad_bucket
        if self.cpu_offload:
            # gradients are exposed on the host next to the shards; the device
            # bucket is copied in by stage_offloaded_gradients() before the step
            if getattr(self, "_host_grad_bucket", None) is None:
                self._host_grad_bucket = torch.zeros(self.bucket_numel, dtype=bucket.dtype,
                                                     pin_memory=torch.cuda.is_available() and bucket.is_cuda)
            bucket = self._host_grad_bucket
        key = bucket.data_ptr()
        for keep, m in zip(part, self.param_metas):
            if not keep:
                m.sharded_param.grad = None
                continue
            # the bucket is persistent, so the DTensor views over it are built once
            # (DTensor construction costs tens of microseconds of host time per call)
            cached = getattr(m, "_grad_view", None)
            if cached is None or cached[0] != key:
                g = bucket.narrow(0, m.bucket_offset, m.padded_numel).view(m.padded_rows, *m.shape[1:])
                local = g.narrow(0, 0, m.local_rows)
                dt = DTensor.from_local(local, device_mesh=self.mesh, placements=(Shard(0),), run_check=False,
                                        shape=m.shape, stride=m.stride)
                cached = (key, dt)
                m._grad_view = cached
            m.sharded_param.grad = cached[1]

    def stage_offloaded_gradients(self) -> None:
        """cpu_offload: copy the reduced (and replica-averaged) device gradients
        into the host bucket the ``.grad`` views cover."""
        if self.cpu_offload and self._grad_valid and getattr(self, "_host_grad_bucket", None) is not None:
            self._host_grad_bucket.copy_(self.grad_bucket)

    def zero_grad(self) -> None:
        """Start a new accumulation window (the bucket is reused, not freed)."""
        self._grad_valid = False
        for m in self.param_metas:
            if m.sharded_param is not None:
                m.sharded_param.grad = None

    def grad_shards(self) -> Optional[torch.Tensor]:
        return self.grad_bucket if self._grad_valid else None
