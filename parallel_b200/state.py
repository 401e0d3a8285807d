"""Process state, process-group init and the parallel topology.

``world_size = dp_replicate x dp_shard x tp``; expert parallelism and
sequence parallelism are folded onto the TP ranks (ep == tp, sp in {1, tp});
context / pipeline / expert-tensor parallelism are reserved and rejected.
The physical layout keeps TP ranks adjacent (strides dp_replicate: tp*dp_shard,
tp: 1, dp_shard: tp) so TP traffic stays on neighbouring GPUs.

Same validation rules, mesh strides and RNG seeding policy as the reference
(parallel/parallel/state.py:15-333).
"""
from __future__ import annotations

import os
import random
from datetime import timedelta
from enum import Enum
from typing import Optional

import numpy as np
import torch
import torch.distributed as dist
from torch.distributed.device_mesh import DeviceMesh

from .utils import is_dist_initialized


class Strategies(str, Enum):
    DP_REPLICATE = "dp_replicate"
    DP_SHARD = "dp_shard"
    TP = "tp"
    CP = "cp"
    SP = "sp"
    EP = "ep"
    PP = "pp"


_SUPPORTED_MESH_DIMS = (Strategies.DP_REPLICATE, Strategies.TP, Strategies.DP_SHARD)
_SUPPORTED_MESH_DIM_NAMES = {d.value for d in _SUPPORTED_MESH_DIMS}


class RuntimeState:
    """Process-wide singleton of the launcher's rank environment."""

    _state: dict = {}

    def __init__(self, backend: str | None = None):
        if self.initialized:
            return
        self._state["RANK"] = int(os.environ.get("RANK", 0))
        self._state["WORLD_SIZE"] = int(os.environ.get("WORLD_SIZE", 1))
        self._state["LOCAL_RANK"] = int(os.environ.get("LOCAL_RANK", 0))
        self._state["backend"] = backend

    @property
    def can_log(self):
        return self.world_size <= 1 or self.rank == 0

    @property
    def local_rank(self):
        return self._state.get("LOCAL_RANK", 0)

    @property
    def rank(self):
        return self._state.get("RANK", 0)

    @property
    def world_size(self):
        return self._state.get("WORLD_SIZE", 1)

    @property
    def backend(self):
        return self._state.get("backend", None)

    @property
    def initialized(self):
        return self._state != {}


def init_dist(cfg, timeout_s: float | None = None) -> None:
    """Select the device and initialise the default process group."""
    device = cfg.config.device_type
    assert device, "device needs to be set in config"
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    if device == "cuda":
        torch.cuda.set_device(local_rank)
    world_size = int(os.environ.get("WORLD_SIZE", "1"))
    if world_size > 1 and not is_dist_initialized():
        if cfg.config.backend == "nccl" and device != "cuda":
            raise RuntimeError("nccl needs to be used with cuda devices")
        kw = {}
        if timeout_s is not None:
            kw["timeout"] = timedelta(seconds=timeout_s)
        if device == "cuda":
            kw["device_id"] = torch.device("cuda", local_rank)
        dist.init_process_group(backend=cfg.config.backend, **kw)


class ParallelConfig:
    """Validated parallel sizes plus the device mesh built from them."""

    def __init__(self, cfg):
        conf = cfg.parallel
        self.dp_replicate_size = conf.dp_replicate
        self.dp_shard_size = conf.dp_shard
        self.tp_size = conf.tp
        self.cp_size = conf.cp
        self.sp_size = conf.sp
        self.ep_size = conf.ep
        self.expert_tp_size = conf.get("expert_tp", 1)
        self.pp_size = conf.pp
        self.device_mesh: Optional[DeviceMesh] = None
        self.device_type: Optional[str] = None
        self.rank = dist.get_rank() if is_dist_initialized() else 0
        self.local_rank = int(os.environ.get("LOCAL_RANK", 0))
        self.world_size = dist.get_world_size() if is_dist_initialized() else 1
        self._device = None
        if self.world_size > 1:
            assert is_dist_initialized()
        sizes = {
            "dp_replicate": self.dp_replicate_size, "dp_shard": self.dp_shard_size, "tp": self.tp_size,
            "cp": self.cp_size, "sp": self.sp_size, "ep": self.ep_size, "expert_tp": self.expert_tp_size,
            "pp": self.pp_size,
        }
        invalid = {n: s for n, s in sizes.items() if not isinstance(s, int) or isinstance(s, bool) or s < 1}
        if invalid:
            raise ValueError(f"Parallel dimensions must be positive integers: {invalid}")
        if self.total_size != self.world_size:
            raise ValueError(
                f"Parallel mesh size {self.total_size} does not match distributed world size {self.world_size}"
            )
        if self.sp_size not in (1, self.tp_size):
            raise ValueError("Sequence parallelism reuses the TP ranks and requires sp == 1 or sp == tp")
        unsupported = {n: s for n, s in sizes.items()
                       if n not in _SUPPORTED_MESH_DIM_NAMES and n not in {"ep", "expert_tp", "sp"} and s > 1}
        if unsupported:
            raise NotImplementedError(
                f"Only replicated, sharded, and tensor parallel mesh dimensions are implemented: {unsupported}"
            )
        if self.expert_tp_size != 1:
            raise NotImplementedError("Expert tensor parallelism is not implemented yet; expert_tp must be 1")
        if self.ep_size > 1 and self.tp_size != self.ep_size:
            raise ValueError("Folded expert parallelism requires tp == ep")

    # ---- sizes
    @property
    def dp_size(self):
        return self.dp_replicate_size * self.dp_shard_size

    @property
    def dp_enabled(self):
        return self.dp_size > 1

    @property
    def model_parallel_size(self):
        """Physical size of the rank group shared by attention TP and MoE EP."""
        return max(self.tp_size, self.ep_size)

    @property
    def model_parallel_enabled(self):
        return self.model_parallel_size > 1

    @property
    def is_distributed(self):
        return self.world_size > 1

    @property
    def is_main_process(self):
        return self.rank == 0

    @property
    def data_rank(self):
        return self._mesh_rank(Strategies.DP_REPLICATE) * self.dp_shard_size + self._mesh_rank(Strategies.DP_SHARD)

    @property
    def data_world_size(self):
        return self.dp_size

    @property
    def total_size(self):
        return (self.dp_replicate_size * self.dp_shard_size * self.model_parallel_size * self.cp_size
                * self.pp_size)

    def __repr__(self):
        return (f"ParallelConfig(dp_replicate={self.dp_replicate_size}, dp_shard={self.dp_shard_size}, "
                f"tp={self.tp_size}, cp={self.cp_size}, sp={self.sp_size}, ep={self.ep_size}, "
                f"expert_tp={self.expert_tp_size}, pp={self.pp_size}, total={self.total_size})")

    # ---- mesh
    def get_mesh_dims(self):
        dims = [x for x in self._supported_mesh_dims() if x[1] > 1]
        return tuple(zip(*dims))

    def _supported_mesh_dims(self):
        return [
            (Strategies.DP_REPLICATE, self.dp_replicate_size),
            (Strategies.TP, self.tp_size),
            (Strategies.DP_SHARD, self.dp_shard_size),
        ]

    def _physical_mesh_strides(self, mesh_dim_names):
        strides = {
            Strategies.DP_REPLICATE: self.tp_size * self.dp_shard_size,
            Strategies.TP: 1,
            Strategies.DP_SHARD: self.tp_size,
        }
        return tuple(strides[n] for n in mesh_dim_names)

    def get_mesh_layout(self):
        """(semantic dim names, shape, physical rank strides); TP ranks adjacent."""
        names, shape = tuple(zip(*self._supported_mesh_dims()))
        return names, shape, self._physical_mesh_strides(names)

    def _coord_to_rank(self, coord, strides):
        return sum(i * s for i, s in zip(coord, strides))

    def _physical_mesh(self, names, shape, strides):
        mesh = torch.empty(shape, dtype=torch.int64)
        for coord in np.ndindex(*shape):
            mesh[coord] = self._coord_to_rank(coord, strides)
        return mesh

    def set_device_mesh(self, device_type: str):
        self.device_type = device_type
        if self.total_size == 1:
            self.device_mesh = None
            return None
        names, shape, strides = self.get_mesh_layout()
        mesh = self._physical_mesh(names, shape, strides)
        self.device_mesh = DeviceMesh(device_type, mesh, mesh_dim_names=tuple(n.value for n in names))
        return self.device_mesh

    @property
    def device(self):
        if self._device is None:
            self._device = (torch.device("cuda", self.local_rank) if self.device_type == "cuda"
                            else torch.device("cpu"))
        return self._device

    def _mesh_rank(self, dim_name) -> int:
        name = dim_name.value if isinstance(dim_name, Strategies) else dim_name
        if self.device_mesh is not None and name in self.device_mesh.mesh_dim_names:
            return self.device_mesh.get_local_rank(name)
        return 0

    def group(self, dim_name):
        """The process group of a mesh dimension, or None if the dim is size 1."""
        name = dim_name.value if isinstance(dim_name, Strategies) else dim_name
        if self.device_mesh is None or name not in self.device_mesh.mesh_dim_names:
            return None
        return self.device_mesh.get_group(name)

    def dim_size(self, dim_name) -> int:
        name = dim_name.value if isinstance(dim_name, Strategies) else dim_name
        return {"dp_replicate": self.dp_replicate_size, "dp_shard": self.dp_shard_size,
                "tp": self.tp_size}.get(name, 1)

    # ---- RNG policy
    def model_init_rngs(self, seed: int = 42):
        """TP ranks get different init seeds."""
        init_seed = seed + self._mesh_rank(Strategies.TP)
        torch.manual_seed(init_seed)
        if self.device_type == "cuda":
            torch.cuda.manual_seed_all(init_seed)

    def model_train_rngs(self, seed: int = 42):
        """DP ranks differ (different data); TP ranks of one replica agree."""
        dp_rank = self.data_rank
        pp_rank = self._mesh_rank(Strategies.PP)
        data_seed = seed + dp_rank
        random.seed(data_seed)
        np.random.seed(data_seed)
        torch_seed = seed + dp_rank * 1000 + pp_rank
        torch.manual_seed(torch_seed)
        if self.device_type == "cuda":
            torch.cuda.manual_seed_all(torch_seed)
