"""Training checkpoints: portable full model + exact-topology sharded directories.

File formats are the reference's (parallel/parallel/engine/checkpoint.py:
21-451), so checkpoints interchange:

* portable: one ``torch.save`` of an OrderedDict of CPU tensors (HF keys,
  full shapes, tied weights as one shared tensor), written by global rank 0
  to a temp file then ``os.replace``d;
* sharded directory (``format_version`` 1, kind ``sharded-training-state``):
  ``model-tp-XXXXX-dp-shard-XXXXX.pt`` (model-parallel) or
  ``model-shard-XXXXX.pt`` holding ``{format_version, model, optimizer}``,
  written only by dp_replicate rank 0; ``rank-state-XXXXX.pt`` per rank
  (RNG python/numpy/torch/cuda, dataloader states, grad scaler, scheduler);
  ``manifest.json`` (topology, layout, file lists, resolved config,
  metadata) and a ``COMPLETE`` marker; the temp directory is renamed into
  place atomically.  Errors on any rank are gathered over a gloo control
  group so every rank raises together; loading validates version, kind,
  topology, layout and file sets.
"""
from __future__ import annotations

import copy
import json
import os
import random
import shutil
import uuid
from collections import OrderedDict
from pathlib import Path
from typing import Any, Optional

import numpy as np
import torch
import torch.distributed as dist

from ..state import Strategies

CHECKPOINT_FORMAT_VERSION = 1


def _cpu_tree(v: Any) -> Any:
    if isinstance(v, torch.Tensor):
        return v.detach().to(device="cpu", copy=True)
    if isinstance(v, OrderedDict):
        return OrderedDict((k, _cpu_tree(x)) for k, x in v.items())
    if isinstance(v, dict):
        return {k: _cpu_tree(x) for k, x in v.items()}
    if isinstance(v, tuple):
        return tuple(_cpu_tree(x) for x in v)
    if isinstance(v, list):
        return [_cpu_tree(x) for x in v]
    return copy.deepcopy(v)


def _jsonable(v: Any) -> Any:
    if v is None or isinstance(v, (str, int, float, bool)):
        return v
    if isinstance(v, Path):
        return str(v)
    if isinstance(v, dict):
        return {str(k): _jsonable(x) for k, x in v.items()}
    if isinstance(v, (list, tuple)):
        return [_jsonable(x) for x in v]
    return repr(v)


class CheckpointManager:
    def __init__(self, engine):
        self.engine = engine
        self.control_group = (dist.new_group(backend="gloo")
                              if dist.is_initialized() and dist.is_gloo_available() else None)

    # ------------------------------------------------------------------ topology
    @property
    def wrapper(self):
        mp = getattr(self.engine, "mp_wrapper", None)
        if mp is not None and mp.is_active:
            return mp
        return self.engine.fsdp_wrapper

    @property
    def rank(self) -> int:
        return dist.get_rank() if dist.is_initialized() else 0

    @property
    def world_size(self) -> int:
        return dist.get_world_size() if dist.is_initialized() else 1

    def _mesh_rank(self, dim: Strategies) -> int:
        mesh = self.engine.pconfig.device_mesh
        if mesh is not None and dim.value in (getattr(mesh, "mesh_dim_names", ()) or ()):
            return mesh.get_local_rank(dim.value)
        return 0

    @property
    def shard_rank(self) -> int:
        return self._mesh_rank(Strategies.DP_SHARD)

    @property
    def tp_rank(self) -> int:
        return self._mesh_rank(Strategies.TP)

    @property
    def model_parallel_active(self) -> bool:
        mp = getattr(self.engine, "mp_wrapper", None)
        return mp is not None and mp.is_active

    @property
    def is_model_writer(self) -> bool:
        return self._mesh_rank(Strategies.DP_REPLICATE) == 0

    def _topology(self) -> dict[str, int]:
        pc = self.engine.pconfig
        return {"world_size": self.world_size, "dp_replicate_size": getattr(pc, "dp_replicate_size", 1),
                "dp_shard_size": getattr(pc, "dp_shard_size", 1), "tp_size": getattr(pc, "tp_size", 1),
                "sp_size": getattr(pc, "sp_size", 1), "ep_size": getattr(pc, "ep_size", 1),
                "expert_tp_size": getattr(pc, "expert_tp_size", 1)}

    # ------------------------------------------------------------------ control plane
    def _broadcast_root_object(self, value: Any) -> Any:
        if not dist.is_initialized():
            return value
        payload = [value if self.rank == 0 else None]
        dist.broadcast_object_list(payload, src=0, group=self.control_group)
        return payload[0]

    def _collect_errors(self, local: Optional[str]) -> list[str]:
        if not dist.is_initialized():
            return [local] if local is not None else []
        errs: list = [None] * self.world_size
        dist.all_gather_object(errs, local, group=self.control_group)
        return [e for e in errs if e is not None]

    def _synchronize_collective_phase(self) -> None:
        """Drain subgroup device work before the next world-level collective so
        communicator launch order cannot depend on timing."""
        if not dist.is_initialized():
            return
        dev = torch.device(self.engine.device)
        if dev.type == "cuda":
            torch.cuda.synchronize(dev)
        dist.barrier(group=self.control_group)

    def _resolved_config(self) -> Any:
        cfg = getattr(self.engine, "cfg", None)
        if cfg is None:
            return None
        if hasattr(cfg, "to_container"):
            return _jsonable(cfg.to_container())
        return _jsonable(cfg)

    def _rng_state(self) -> dict:
        st = {"python": random.getstate(), "numpy": np.random.get_state(), "torch": torch.get_rng_state()}
        if torch.device(self.engine.device).type == "cuda":
            st["cuda"] = torch.cuda.get_rng_state(self.engine.device)
        return st

    def _restore_rng_state(self, st: dict) -> None:
        random.setstate(st["python"])
        np.random.set_state(st["numpy"])
        torch.set_rng_state(st["torch"])
        if "cuda" in st:
            torch.cuda.set_rng_state(st["cuda"], self.engine.device)

    # ------------------------------------------------------------------ state dicts
    def full_state_dict(self):
        st = self.wrapper.full_state_dict()
        self._synchronize_collective_phase()
        return st

    def load_full_state_dict(self, state_dict, strict: bool = True):
        res = self.wrapper.load_full_state_dict(state_dict, strict=strict)
        self._synchronize_collective_phase()
        return res

    def sharded_state_dict(self) -> dict:
        return self.wrapper.sharded_state_dict()

    def load_sharded_state_dict(self, state_dict, strict: bool = True):
        return self.wrapper.load_sharded_state_dict(state_dict, strict=strict)

    # ------------------------------------------------------------------ portable model
    def save_full_model(self, path) -> None:
        """Portable CPU state dict (every rank must call)."""
        path = Path(path)
        state = self.full_state_dict()
        res = None
        if self.rank == 0:
            tmp = path.with_name(f".{path.name}.tmp-{uuid.uuid4().hex}")
            try:
                if path.exists():
                    raise FileExistsError(f"Checkpoint already exists: {path}")
                path.parent.mkdir(parents=True, exist_ok=True)
                torch.save(state, tmp)
                os.replace(tmp, path)
                res = {"error": None}
            except Exception as e:
                if tmp.exists():
                    tmp.unlink()
                res = {"error": f"{type(e).__name__}: {e}"}
        res = self._broadcast_root_object(res)
        if res["error"] is not None:
            raise RuntimeError(f"Failed to save full model: {res['error']}")

    def load_full_model(self, path, strict: bool = True):
        state, res = None, None
        if self.rank == 0:
            try:
                state = torch.load(Path(path), map_location="cpu", weights_only=False)
                res = {"error": None}
            except Exception as e:
                res = {"error": f"{type(e).__name__}: {e}"}
        res = self._broadcast_root_object(res)
        if res["error"] is not None:
            raise RuntimeError(f"Failed to load full model: {res['error']}")
        return self.load_full_state_dict(state, strict=strict)

    # ------------------------------------------------------------------ sharded directory
    def _prepare_checkpoint_directory(self, path: Path) -> Path:
        res = None
        if self.rank == 0:
            try:
                if path.exists():
                    raise FileExistsError(f"Checkpoint already exists: {path}")
                path.parent.mkdir(parents=True, exist_ok=True)
                tmp = path.with_name(f".{path.name}.tmp-{uuid.uuid4().hex}")
                tmp.mkdir()
                res = {"path": str(tmp), "error": None}
            except Exception as e:
                res = {"path": None, "error": f"{type(e).__name__}: {e}"}
        res = self._broadcast_root_object(res)
        if res["error"] is not None:
            raise RuntimeError(f"Failed to initialize checkpoint: {res['error']}")
        return Path(res["path"])

    def _model_file_name(self, shard_rank: int, tp_rank: int | None = None) -> str:
        if self.model_parallel_active:
            tp_rank = self.tp_rank if tp_rank is None else tp_rank
            return f"model-tp-{tp_rank:05d}-dp-shard-{shard_rank:05d}.pt"
        return f"model-shard-{shard_rank:05d}.pt"

    def _model_file_names(self) -> list[str]:
        t = self._topology()
        if self.model_parallel_active:
            return [self._model_file_name(s, r) for r in range(t["tp_size"]) for s in range(t["dp_shard_size"])]
        return [self._model_file_name(s) for s in range(t["dp_shard_size"])]

    def _rank_file_name(self, rank: int) -> str:
        return f"rank-state-{rank:05d}.pt"

    def save(self, path, *, step: int, dataloader_state=None, eval_dataloader_state=None, metadata=None) -> None:
        """Atomically save an exact-resume, same-topology sharded checkpoint."""
        self._synchronize_collective_phase()
        path = Path(path)
        tmp = self._prepare_checkpoint_directory(path)
        local_error = None
        try:
            if self.is_model_writer:
                payload = {"format_version": CHECKPOINT_FORMAT_VERSION, "model": self.sharded_state_dict(),
                           "optimizer": _cpu_tree(self.engine.optimizer.state_dict())}
                torch.save(payload, tmp / self._model_file_name(self.shard_rank, self.tp_rank))
            scaler = getattr(self.engine, "grad_scaler", None)
            scheduler = getattr(self.engine, "scheduler", None)
            rank_payload = {
                "format_version": CHECKPOINT_FORMAT_VERSION, "rank": self.rank, "rng": self._rng_state(),
                "dataloader": copy.deepcopy(dataloader_state), "eval_dataloader": copy.deepcopy(eval_dataloader_state),
                "grad_scaler": scaler.state_dict() if scaler is not None else None,
                "scheduler": scheduler.state_dict() if scheduler is not None else None,
            }
            torch.save(rank_payload, tmp / self._rank_file_name(self.rank))
        except Exception as e:
            local_error = f"rank {self.rank}: {type(e).__name__}: {e}"
        errors = self._collect_errors(local_error)
        if errors:
            if self.rank == 0:
                shutil.rmtree(tmp, ignore_errors=True)
            raise RuntimeError("Failed to write checkpoint: " + " | ".join(errors))
        res = None
        if self.rank == 0:
            try:
                manifest = {
                    "format_version": CHECKPOINT_FORMAT_VERSION, "kind": "sharded-training-state", "step": int(step),
                    "topology": self._topology(), "layout": self.wrapper.checkpoint_layout(),
                    "model_files": self._model_file_names(),
                    "rank_files": [self._rank_file_name(r) for r in range(self.world_size)],
                    "config": self._resolved_config(), "metadata": _jsonable(metadata or {}),
                }
                (tmp / "manifest.json").write_text(json.dumps(manifest, indent=2, sort_keys=True) + "\n",
                                                   encoding="utf-8")
                (tmp / "COMPLETE").write_text("complete\n", encoding="utf-8")
                os.replace(tmp, path)
                res = {"error": None}
            except Exception as e:
                shutil.rmtree(tmp, ignore_errors=True)
                res = {"error": f"{type(e).__name__}: {e}"}
        res = self._broadcast_root_object(res)
        if res["error"] is not None:
            raise RuntimeError(f"Failed to finalize checkpoint: {res['error']}")

    def _read_manifest(self, path: Path) -> dict:
        res = None
        if self.rank == 0:
            try:
                if not (path / "COMPLETE").is_file():
                    raise RuntimeError("Checkpoint has no COMPLETE marker")
                res = {"manifest": json.loads((path / "manifest.json").read_text(encoding="utf-8")), "error": None}
            except Exception as e:
                res = {"manifest": None, "error": f"{type(e).__name__}: {e}"}
        res = self._broadcast_root_object(res)
        if res["error"] is not None:
            raise RuntimeError(f"Failed to read checkpoint: {res['error']}")
        return res["manifest"]

    def load(self, path, *, strict: bool = True) -> dict:
        """Restore model, optimizer, scaler, scheduler, RNG and data position."""
        path = Path(path)
        manifest = self._read_manifest(path)
        if manifest.get("format_version") != CHECKPOINT_FORMAT_VERSION:
            raise RuntimeError(f"Unsupported checkpoint version: {manifest.get('format_version')}")
        if manifest.get("kind") != "sharded-training-state":
            raise RuntimeError(f"Unsupported checkpoint kind: {manifest.get('kind')}")
        if manifest.get("topology") != self._topology():
            raise RuntimeError("Checkpoint topology does not match the current distributed topology: "
                               f"saved={manifest.get('topology')}, current={self._topology()}")
        if manifest.get("layout") != self.wrapper.checkpoint_layout():
            raise RuntimeError("Checkpoint model layout does not match the current model")
        if manifest.get("model_files") != self._model_file_names():
            raise RuntimeError("Checkpoint manifest has an invalid model file set")
        if manifest.get("rank_files") != [self._rank_file_name(r) for r in range(self.world_size)]:
            raise RuntimeError("Checkpoint manifest has an invalid rank-state file set")
        local_error, rank_payload = None, None
        try:
            mp = torch.load(path / self._model_file_name(self.shard_rank, self.tp_rank), map_location="cpu",
                            weights_only=False)
            if mp.get("format_version") != CHECKPOINT_FORMAT_VERSION:
                raise RuntimeError("Model shard has an unsupported format version")
            rank_payload = torch.load(path / self._rank_file_name(self.rank), map_location="cpu", weights_only=False)
            if rank_payload.get("format_version") != CHECKPOINT_FORMAT_VERSION:
                raise RuntimeError("Rank state has an unsupported format version")
            if rank_payload.get("rank") != self.rank:
                raise RuntimeError(f"Loaded rank state for {rank_payload.get('rank')} on rank {self.rank}")
            rng = rank_payload.get("rng")
            if not isinstance(rng, dict) or not {"python", "numpy", "torch"}.issubset(rng):
                raise RuntimeError("Rank state has incomplete RNG state")
            if torch.device(self.engine.device).type == "cuda" and "cuda" not in rng:
                raise RuntimeError("Rank state has no CUDA RNG state")
            scaler = getattr(self.engine, "grad_scaler", None)
            scheduler = getattr(self.engine, "scheduler", None)
            if (scaler is None) != (rank_payload.get("grad_scaler") is None):
                raise RuntimeError("Checkpoint grad-scaler configuration does not match")
            if (scheduler is None) != (rank_payload.get("scheduler") is None):
                raise RuntimeError("Checkpoint scheduler configuration does not match")
            self.load_sharded_state_dict(mp["model"], strict=strict)
            self.engine.optimizer.load_state_dict(mp["optimizer"])
            if scaler is not None:
                scaler.load_state_dict(rank_payload["grad_scaler"])
            if scheduler is not None:
                scheduler.load_state_dict(rank_payload["scheduler"])
        except Exception as e:
            local_error = f"rank {self.rank}: {type(e).__name__}: {e}"
        errors = self._collect_errors(local_error)
        if errors:
            raise RuntimeError("Failed to load checkpoint: " + " | ".join(errors))
        self._restore_rng_state(rank_payload["rng"])
        return {"step": manifest["step"], "dataloader_state": rank_payload.get("dataloader"),
                "eval_dataloader_state": rank_payload.get("eval_dataloader"),
                "metadata": manifest.get("metadata", {}), "config": manifest.get("config")}
