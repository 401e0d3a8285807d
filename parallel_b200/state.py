"""Launch environment, process-group start-up and the parallel topology.

Topology rules (behaviour of the reference's ``parallel/parallel/state.py:
15-333``, which checkpoints, data sharding and RNG streams depend on):

* ``world = dp_replicate x dp_shard x tp``.  Expert parallelism and sequence
  parallelism run on the TP ranks (``ep == tp``, ``sp in {1, tp}``); context
  parallelism, pipeline parallelism and expert-tensor parallelism are
  reserved keys that must stay 1.
* The device mesh has the named dimensions (dp_replicate, tp, dp_shard) in
  that order, but ranks are laid out TP-innermost: global rank =
  r * (tp * dp_shard) + s * tp + t for replica r, shard s, TP rank t, so a
  TP group is a block of neighbouring GPUs.
* RNG: model initialisation seeds ``seed + tp_rank``; training seeds python /
  numpy with ``seed + data_rank`` and torch with ``seed + 1000 * data_rank +
  pp_rank``, so TP ranks of one replica draw identical streams.

The table ``_DIMENSIONS`` drives validation, the mesh and the size
accessors; each rule of ``_RULES`` is one check with its own message.
"""
from __future__ import annotations

import os
import random
from dataclasses import dataclass
from datetime import timedelta
from enum import Enum
from typing import Callable, Optional

import numpy as np
import torch
import torch.distributed as dist
from torch.distributed.device_mesh import DeviceMesh

from .utils import is_dist_initialized


class Strategies(str, Enum):
    """Names of the parallel dimensions (also the device-mesh dim names)."""

    DP_REPLICATE = "dp_replicate"
    DP_SHARD = "dp_shard"
    TP = "tp"
    CP = "cp"
    SP = "sp"
    EP = "ep"
    PP = "pp"


# --------------------------------------------------------------------------- launch environment
@dataclass(frozen=True)
class LaunchEnv:
    """The launcher's rank variables (torchrun / mp.spawn), read once."""

    rank: int
    world_size: int
    local_rank: int
    backend: Optional[str]

    @classmethod
    def from_environ(cls, backend: Optional[str] = None) -> "LaunchEnv":
        env = os.environ
        return cls(int(env.get("RANK", 0)), int(env.get("WORLD_SIZE", 1)), int(env.get("LOCAL_RANK", 0)), backend)

    @property
    def can_log(self) -> bool:
        return self.world_size <= 1 or self.rank == 0


_LAUNCH: Optional[LaunchEnv] = None


def RuntimeState(backend: Optional[str] = None) -> LaunchEnv:  # noqa: N802 (kept as the public name)
    """The process's ``LaunchEnv``; the first call (optionally naming the
    backend) fixes it for the life of the process."""
    global _LAUNCH
    if _LAUNCH is None:
        _LAUNCH = LaunchEnv.from_environ(backend)
    return _LAUNCH


def reset_runtime_state() -> None:
    """Forget the cached launch environment (tests)."""
    global _LAUNCH
    _LAUNCH = None


def init_dist(cfg, timeout_s: float | None = None) -> None:
    """Bind this process to its GPU and start the default process group (env
    rendezvous) when the launcher started more than one rank."""
    device = cfg.config.device_type
    if not device:
        raise ValueError("config.device_type must be set (cuda or cpu)")
    env = LaunchEnv.from_environ(cfg.config.backend)
    if device == "cuda":
        torch.cuda.set_device(env.local_rank)
    if env.world_size <= 1 or is_dist_initialized():
        return
    if env.backend == "nccl" and device != "cuda":
        raise RuntimeError(f"the nccl backend drives CUDA devices; config.device_type is {device!r}")
    options = {}
    if timeout_s is not None:
        options["timeout"] = timedelta(seconds=timeout_s)
    if device == "cuda":
        options["device_id"] = torch.device("cuda", env.local_rank)
    dist.init_process_group(backend=env.backend, **options)


# --------------------------------------------------------------------------- topology table
@dataclass(frozen=True)
class _Dim:
    strategy: Strategies
    attr: str                # ParallelConfig attribute holding the size
    role: str                # "mesh": own mesh dim; "folded": on the TP ranks; "reserved": must be 1


_DIMENSIONS = (
    _Dim(Strategies.DP_REPLICATE, "dp_replicate_size", "mesh"),
    _Dim(Strategies.DP_SHARD, "dp_shard_size", "mesh"),
    _Dim(Strategies.TP, "tp_size", "mesh"),
    _Dim(Strategies.CP, "cp_size", "reserved"),
    _Dim(Strategies.SP, "sp_size", "folded"),
    _Dim(Strategies.EP, "ep_size", "folded"),
    _Dim(Strategies.PP, "pp_size", "reserved"),
)
_MESH_ORDER = (Strategies.DP_REPLICATE, Strategies.TP, Strategies.DP_SHARD)


def _size_rule(c: "ParallelConfig"):
    bad = {k: v for k, v in c.sizes().items() if type(v) is not int or v < 1}
    if bad:
        return ValueError(f"parallel sizes must be positive integers; got {bad}")


def _world_rule(c: "ParallelConfig"):
    if c.total_size != c.world_size:
        return ValueError(f"the parallel layout covers {c.total_size} ranks, which does not match the "
                          f"{c.world_size} ranks of this job")


def _sp_rule(c: "ParallelConfig"):
    if c.sp_size not in (1, c.tp_size):
        return ValueError(f"sequence parallelism runs on the TP ranks, so it needs sp == 1 or sp == tp "
                          f"(sp={c.sp_size}, tp={c.tp_size})")


def _reserved_rule(c: "ParallelConfig"):
    on = {d.strategy.value: getattr(c, d.attr) for d in _DIMENSIONS
          if d.role == "reserved" and getattr(c, d.attr) > 1}
    if on:
        return NotImplementedError(f"{on}: only data (replicate / shard) and tensor parallel dimensions, with "
                                   "EP and SP on the TP ranks, are built")


def _expert_tp_rule(c: "ParallelConfig"):
    if c.expert_tp_size != 1:
        return NotImplementedError(f"expert_tp={c.expert_tp_size}: experts are not tensor-parallel here, "
                                   "expert_tp must be 1")


def _ep_rule(c: "ParallelConfig"):
    if c.ep_size > 1 and c.ep_size != c.tp_size:
        return ValueError(f"expert parallelism runs on the TP ranks and needs tp == ep (tp={c.tp_size}, "
                          f"ep={c.ep_size})")


_RULES: tuple[Callable[["ParallelConfig"], Optional[Exception]], ...] = (
    _size_rule, _world_rule, _sp_rule, _reserved_rule, _expert_tp_rule, _ep_rule)


class ParallelConfig:
    """Validated parallel sizes of ``cfg.parallel`` plus the device mesh."""

    def __init__(self, cfg):
        section = cfg.parallel
        for d in _DIMENSIONS:
            setattr(self, d.attr, section.get(d.strategy.value, 1) if hasattr(section, "get")
                    else getattr(section, d.strategy.value))
        self.expert_tp_size = section.get("expert_tp", 1) if hasattr(section, "get") else 1
        self.device_mesh: Optional[DeviceMesh] = None
        self.device_type: Optional[str] = None
        self._device = None
        joined = is_dist_initialized()
        self.rank = dist.get_rank() if joined else 0
        self.world_size = dist.get_world_size() if joined else 1
        self.local_rank = int(os.environ.get("LOCAL_RANK", 0))
        if self.world_size > 1 and not joined:
            raise RuntimeError("a multi-rank job needs the process group started (init_dist) first")
        for rule in _RULES:
            problem = rule(self)
            if problem is not None:
                raise problem

    def sizes(self) -> dict:
        out = {d.strategy.value: getattr(self, d.attr) for d in _DIMENSIONS}
        out["expert_tp"] = self.expert_tp_size
        return out

    # ------------------------------------------------------------------ derived sizes
    @property
    def model_parallel_size(self) -> int:
        """Ranks of one TP group (shared by attention TP and MoE EP)."""
        return max(self.tp_size, self.ep_size)

    @property
    def model_parallel_enabled(self) -> bool:
        return self.model_parallel_size > 1

    @property
    def dp_size(self) -> int:
        return self.dp_replicate_size * self.dp_shard_size

    @property
    def dp_enabled(self) -> bool:
        return self.dp_size > 1

    @property
    def data_world_size(self) -> int:
        return self.dp_size

    @property
    def total_size(self) -> int:
        return self.dp_size * self.model_parallel_size * self.cp_size * self.pp_size

    @property
    def is_distributed(self) -> bool:
        return self.world_size > 1

    @property
    def is_main_process(self) -> bool:
        return self.rank == 0

    @property
    def data_rank(self) -> int:
        """Index of this rank's data stream (TP ranks of a replica share it)."""
        return self._mesh_rank(Strategies.DP_REPLICATE) * self.dp_shard_size + self._mesh_rank(Strategies.DP_SHARD)

    def __repr__(self) -> str:
        body = ", ".join(f"{k}={v}" for k, v in self.sizes().items())
        return f"ParallelConfig({body}, total={self.total_size})"

    # ------------------------------------------------------------------ mesh
    def _mesh_sizes(self) -> dict:
        return {Strategies.DP_REPLICATE: self.dp_replicate_size, Strategies.TP: self.tp_size,
                Strategies.DP_SHARD: self.dp_shard_size}

    def _rank_strides(self) -> dict:
        """Global-rank step of each mesh dimension (TP innermost)."""
        return {Strategies.TP: 1, Strategies.DP_SHARD: self.tp_size,
                Strategies.DP_REPLICATE: self.tp_size * self.dp_shard_size}

    def get_mesh_layout(self):
        """(dim names, sizes, physical rank strides) in mesh order."""
        sizes, strides = self._mesh_sizes(), self._rank_strides()
        return _MESH_ORDER, tuple(sizes[d] for d in _MESH_ORDER), tuple(strides[d] for d in _MESH_ORDER)

    def get_mesh_dims(self):
        """(names, sizes) of the mesh dimensions larger than 1."""
        sizes = self._mesh_sizes()
        return tuple(zip(*[(d, sizes[d]) for d in _MESH_ORDER if sizes[d] > 1]))

    def _physical_mesh(self, names, shape, strides) -> torch.Tensor:
        """Global rank at every mesh coordinate: sum over dims of index x stride."""
        table = np.zeros(shape, dtype=np.int64)
        for axis, (size, stride) in enumerate(zip(shape, strides)):
            index_shape = [1] * len(shape)
            index_shape[axis] = size
            table = table + np.arange(size, dtype=np.int64).reshape(index_shape) * stride
        return torch.from_numpy(table)

    def set_device_mesh(self, device_type: str):
        self.device_type = device_type
        if self.total_size == 1:
            self.device_mesh = None
            return None
        names, shape, strides = self.get_mesh_layout()
        self.device_mesh = DeviceMesh(device_type, self._physical_mesh(names, shape, strides),
                                      mesh_dim_names=tuple(d.value for d in names))
        return self.device_mesh

    @property
    def device(self) -> torch.device:
        if self._device is None:
            self._device = (torch.device("cuda", self.local_rank) if self.device_type == "cuda"
                            else torch.device("cpu"))
        return self._device

    def _mesh_rank(self, dim) -> int:
        name = Strategies(dim).value
        mesh = self.device_mesh
        if mesh is None or name not in (mesh.mesh_dim_names or ()):
            return 0
        return mesh.get_local_rank(name)

    def group(self, dim):
        """Process group of a mesh dimension, or None where it has size 1."""
        name = Strategies(dim).value
        mesh = self.device_mesh
        if mesh is None or name not in (mesh.mesh_dim_names or ()):
            return None
        return mesh.get_group(name)

    def dim_size(self, dim) -> int:
        return self._mesh_sizes().get(Strategies(dim), 1)

    # ------------------------------------------------------------------ RNG policy
    def _seed_all(self, torch_seed: int, host_seed: Optional[int] = None) -> None:
        if host_seed is not None:
            random.seed(host_seed)
            np.random.seed(host_seed)
        torch.manual_seed(torch_seed)
        if self.device_type == "cuda":
            torch.cuda.manual_seed_all(torch_seed)

    def model_init_rngs(self, seed: int = 42) -> None:
        """Initialisation draws differ between TP ranks (each builds its own shards)."""
        self._seed_all(seed + self._mesh_rank(Strategies.TP))

    def model_train_rngs(self, seed: int = 42) -> None:
        """Training draws differ between data streams and agree within a TP group."""
        data = self.data_rank
        self._seed_all(seed + 1000 * data + self._mesh_rank(Strategies.PP), host_seed=seed + data)
