"""Training checkpoints: a portable full model file and exact-topology directories.

The on-disk formats are an interface shared with the reference
(``parallel/parallel/engine/checkpoint.py:21-451``), so checkpoints written by
either implementation load in the other:

* portable model: one ``torch.save`` of an ordered dict of full CPU tensors
  (HF parameter names; tied weights stay one shared tensor);
* exact-topology directory, ``format_version`` 1, ``kind``
  ``"sharded-training-state"``:

  - ``model-tp-TTTTT-dp-shard-SSSSS.pt`` (model parallel) or
    ``model-shard-SSSSS.pt``: ``{"format_version", "model", "optimizer"}``,
    written by the dp_replicate-0 copy of each shard only;
  - ``rank-state-RRRRR.pt`` per rank: ``{"format_version", "rank", "rng",
    "dataloader", "eval_dataloader", "grad_scaler", "scheduler"}``;
  - ``manifest.json`` (topology, layout, file lists, resolved config, user
    metadata) and a ``COMPLETE`` marker.

How it is organised here:

* ``_ControlPlane`` runs every decision that must come out the same on all
  ranks over a gloo group: an action on the root whose outcome (value or
  error text) is broadcast, or an action on every rank whose failures are
  gathered, so a failure anywhere raises on every rank together.
* ``DirectoryLayout`` is the single place that knows the file names.
* ``_MANIFEST_SCHEMA`` is a declarative table: saving fills the manifest from
  the same expectations that loading checks; ``_check_rank_state`` is the
  table of rank-file checks.
* RNG capture / restore walks one table of generator sources.

The directory is assembled under a hidden sibling and renamed into place
only after every file and the marker exist.
"""
from __future__ import annotations

import copy
import json
import os
import random
import shutil
import uuid
from dataclasses import dataclass
from pathlib import Path
from typing import Any, Callable, Optional

import numpy as np
import torch
import torch.distributed as dist
from torch.utils._pytree import tree_map

from ..state import Strategies

CHECKPOINT_FORMAT_VERSION = 1
CHECKPOINT_KIND = "sharded-training-state"


class CheckpointError(RuntimeError):
    """Raised on every rank when any rank failed a checkpoint phase."""


# --------------------------------------------------------------------------- value helpers
def host_copy(tree: Any) -> Any:
    """Detached CPU copies of every tensor in a nested container; every other
    leaf is deep-copied, so the result shares nothing with live state."""
    return tree_map(lambda leaf: leaf.detach().to("cpu", copy=True) if isinstance(leaf, torch.Tensor)
                    else copy.deepcopy(leaf), tree)


def json_safe(value: Any) -> Any:
    """Plain JSON data for a config / metadata tree: containers become dicts
    with string keys and lists, paths become strings, and anything JSON has no
    type for becomes its ``repr``."""
    if isinstance(value, dict):
        return {str(k): json_safe(v) for k, v in value.items()}
    if isinstance(value, (list, tuple)):
        return [json_safe(v) for v in value]
    if isinstance(value, os.PathLike):
        return os.fspath(value)
    if value is None or isinstance(value, (bool, int, float, str)):
        return value
    return repr(value)


# --------------------------------------------------------------------------- RNG sources
_HOST_RNG_SOURCES: dict[str, tuple[Callable[[], Any], Callable[[Any], None]]] = {
    "python": (random.getstate, random.setstate),
    "numpy": (np.random.get_state, np.random.set_state),
    "torch": (torch.get_rng_state, torch.set_rng_state),
}


def _rng_sources(device: torch.device) -> dict:
    sources = dict(_HOST_RNG_SOURCES)
    if device.type == "cuda":
        sources["cuda"] = (lambda: torch.cuda.get_rng_state(device), lambda s: torch.cuda.set_rng_state(s, device))
    return sources


# --------------------------------------------------------------------------- control plane
class _ControlPlane:
    """Host-side agreement between ranks (gloo; a no-op without a process group)."""

    def __init__(self):
        self.distributed = dist.is_initialized()
        self.group = dist.new_group(backend="gloo") if self.distributed and dist.is_gloo_available() else None
        self.rank = dist.get_rank() if self.distributed else 0
        self.world = dist.get_world_size() if self.distributed else 1

    def on_root(self, phase: str, action: Callable[[], Any]) -> Any:
        """Run ``action`` on global rank 0 and hand its result to every rank;
        if it raised, every rank raises ``CheckpointError`` naming ``phase``."""
        outcome = None
        if self.rank == 0:
            try:
                outcome = ("ok", action())
            except Exception as exc:  # reported on every rank below
                outcome = ("error", f"{type(exc).__name__}: {exc}")
        if self.distributed:
            box = [outcome]
            dist.broadcast_object_list(box, src=0, group=self.group)
            outcome = box[0]
        status, payload = outcome
        if status != "ok":
            raise CheckpointError(f"checkpoint {phase} failed: {payload}")
        return payload

    def on_every_rank(self, phase: str, action: Callable[[], Any],
                      cleanup: Optional[Callable[[], None]] = None) -> Any:
        """Run ``action`` on each rank; if any rank raised, every rank raises a
        ``CheckpointError`` listing each failing rank (``cleanup`` runs first,
        on rank 0)."""
        result, failure = None, None
        try:
            result = action()
        except Exception as exc:
            failure = f"rank {self.rank}: {type(exc).__name__}: {exc}"
        failures = [failure]
        if self.distributed:
            failures = [None] * self.world
            dist.all_gather_object(failures, failure, group=self.group)
        failures = [f for f in failures if f is not None]
        if failures:
            if cleanup is not None and self.rank == 0:
                cleanup()
            raise CheckpointError(f"checkpoint {phase} failed: " + " | ".join(failures))
        return result

    def fence(self, device: torch.device) -> None:
        """Finish this rank's queued device work, then meet every rank.

        Checkpoint phases issue collectives on several disjoint NCCL groups
        (TP, dp_shard, dp_replicate); draining the device before the next
        world-level step keeps the launch order of communicators independent
        of timing."""
        if not self.distributed:
            return
        if device.type == "cuda":
            torch.cuda.synchronize(device)
        dist.barrier(group=self.group)


# --------------------------------------------------------------------------- directory layout
@dataclass(frozen=True)
class DirectoryLayout:
    """File names of one exact-topology checkpoint directory."""

    world_size: int
    tp_size: int
    dp_shard_size: int
    model_parallel: bool

    def model_file(self, shard_rank: int, tp_rank: int) -> str:
        if self.model_parallel:
            return f"model-tp-{tp_rank:05d}-dp-shard-{shard_rank:05d}.pt"
        return f"model-shard-{shard_rank:05d}.pt"

    def model_files(self) -> list[str]:
        tp_ranks = range(self.tp_size) if self.model_parallel else range(1)
        return [self.model_file(s, t) for t in tp_ranks for s in range(self.dp_shard_size)]

    @staticmethod
    def rank_file(rank: int) -> str:
        return f"rank-state-{rank:05d}.pt"

    def rank_files(self) -> list[str]:
        return [self.rank_file(r) for r in range(self.world_size)]


# --------------------------------------------------------------------------- schemas
# (manifest key, how the current job computes it, what a mismatch means).  The
# same table fills the manifest on save and validates it on load.
_MANIFEST_SCHEMA: list[tuple[str, Callable[["CheckpointManager"], Any], str]] = [
    ("format_version", lambda m: CHECKPOINT_FORMAT_VERSION,
     "checkpoint format_version {saved!r} is not supported (this build reads {current!r})"),
    ("kind", lambda m: CHECKPOINT_KIND, "checkpoint kind {saved!r} is not {current!r}"),
    ("topology", lambda m: m.topology(),
     "checkpoint topology does not match this job: saved {saved}, running {current}"),
    ("layout", lambda m: m.wrapper.checkpoint_layout(),
     "checkpoint model layout does not match the model being restored"),
    ("model_files", lambda m: m.layout().model_files(),
     "checkpoint manifest lists model files {saved} where this topology expects {current}"),
    ("rank_files", lambda m: m.layout().rank_files(),
     "checkpoint manifest lists rank-state files {saved} where this topology expects {current}"),
]


def _check_rank_state(payload: dict, rank: int, device: torch.device, has_scaler: bool,
                      has_scheduler: bool) -> None:
    rng = payload.get("rng")
    problems = [
        (payload.get("format_version") != CHECKPOINT_FORMAT_VERSION,
         f"rank-state format_version {payload.get('format_version')!r} is not supported"),
        (payload.get("rank") != rank, f"rank-state file of rank {payload.get('rank')!r} opened by rank {rank}"),
        (not isinstance(rng, dict) or not set(_HOST_RNG_SOURCES) <= set(rng),
         "rank state has incomplete RNG state (python, numpy and torch are required)"),
        (device.type == "cuda" and isinstance(rng, dict) and "cuda" not in rng,
         "rank state has incomplete RNG state (no CUDA generator state for a CUDA job)"),
        (has_scaler != (payload.get("grad_scaler") is not None),
         "grad scaler present in only one of the checkpoint and this job"),
        (has_scheduler != (payload.get("scheduler") is not None),
         "LR scheduler present in only one of the checkpoint and this job"),
    ]
    for failed, message in problems:
        if failed:
            raise ValueError(message)


# --------------------------------------------------------------------------- manager
class CheckpointManager:
    """Portable and exact-topology checkpoints of one ``ParallelEngine``."""

    def __init__(self, engine):
        self.engine = engine
        self.plane = _ControlPlane()

    # ------------------------------------------------------------------ job description
    @property
    def device(self) -> torch.device:
        return torch.device(self.engine.device)

    @property
    def rank(self) -> int:
        return self.plane.rank

    @property
    def world_size(self) -> int:
        return self.plane.world

    @property
    def model_parallel_active(self) -> bool:
        mp = getattr(self.engine, "mp_wrapper", None)
        return mp is not None and mp.is_active

    @property
    def wrapper(self):
        """The object owning the model's state dicts (model-parallel wrapper if
        active, else the FSDP wrapper, which is a pass-through without FSDP)."""
        return self.engine.mp_wrapper if self.model_parallel_active else self.engine.fsdp_wrapper

    def coordinate(self, dim: Strategies) -> int:
        mesh = self.engine.pconfig.device_mesh
        names = tuple(getattr(mesh, "mesh_dim_names", None) or ()) if mesh is not None else ()
        return mesh.get_local_rank(dim.value) if dim.value in names else 0

    def topology(self) -> dict[str, int]:
        pc = self.engine.pconfig
        sizes = {key: getattr(pc, key, 1) for key in
                 ("dp_replicate_size", "dp_shard_size", "tp_size", "sp_size", "ep_size", "expert_tp_size")}
        return {"world_size": self.world_size, **sizes}

    def layout(self) -> DirectoryLayout:
        t = self.topology()
        return DirectoryLayout(self.world_size, t["tp_size"], t["dp_shard_size"], self.model_parallel_active)

    def _my_model_file(self) -> str:
        return self.layout().model_file(self.coordinate(Strategies.DP_SHARD), self.coordinate(Strategies.TP))

    # ------------------------------------------------------------------ state dicts
    def full_state_dict(self):
        state = self.wrapper.full_state_dict()
        self.plane.fence(self.device)
        return state

    def load_full_state_dict(self, state_dict, strict: bool = True):
        result = self.wrapper.load_full_state_dict(state_dict, strict=strict)
        self.plane.fence(self.device)
        return result

    def sharded_state_dict(self) -> dict:
        return self.wrapper.sharded_state_dict()

    def load_sharded_state_dict(self, state_dict, strict: bool = True):
        return self.wrapper.load_sharded_state_dict(state_dict, strict=strict)

    # ------------------------------------------------------------------ portable file
    def save_full_model(self, path) -> None:
        """Write the portable full model (collective: every rank calls it)."""
        target = Path(path)
        state = self.full_state_dict()

        def write():
            if target.exists():
                raise FileExistsError(f"Checkpoint already exists: {target}")
            target.parent.mkdir(parents=True, exist_ok=True)
            partial = target.with_name(f".{target.name}.partial-{uuid.uuid4().hex}")
            try:
                torch.save(state, partial)
                os.replace(partial, target)
            finally:
                partial.unlink(missing_ok=True)

        self.plane.on_root("full-model save", write)

    def load_full_model(self, path, strict: bool = True):
        """Read the portable file on rank 0 and distribute it through the
        wrapper's ``load_full_state_dict`` (collective)."""
        holder = {}

        def read():
            holder["state"] = torch.load(Path(path), map_location="cpu", weights_only=False)

        self.plane.on_root("full-model load", read)
        return self.load_full_state_dict(holder.get("state"), strict=strict)

    # ------------------------------------------------------------------ exact-topology directory
    def _engine_extras(self) -> tuple[Any, Any]:
        return getattr(self.engine, "grad_scaler", None), getattr(self.engine, "scheduler", None)

    def _resolved_config(self) -> Any:
        cfg = getattr(self.engine, "cfg", None)
        if cfg is None:
            return None
        return json_safe(cfg.to_container() if hasattr(cfg, "to_container") else cfg)

    def _write_my_files(self, staging: Path, dataloader_state, eval_dataloader_state) -> None:
        if self.coordinate(Strategies.DP_REPLICATE) == 0:  # one copy of each shard
            torch.save({"format_version": CHECKPOINT_FORMAT_VERSION,
                        "model": self.sharded_state_dict(),
                        "optimizer": host_copy(self.engine.optimizer.state_dict())},
                       staging / self._my_model_file())
        scaler, scheduler = self._engine_extras()
        torch.save({"format_version": CHECKPOINT_FORMAT_VERSION,
                    "rank": self.rank,
                    "rng": {name: get() for name, (get, _) in _rng_sources(self.device).items()},
                    "dataloader": copy.deepcopy(dataloader_state),
                    "eval_dataloader": copy.deepcopy(eval_dataloader_state),
                    "grad_scaler": None if scaler is None else scaler.state_dict(),
                    "scheduler": None if scheduler is None else scheduler.state_dict()},
                   staging / DirectoryLayout.rank_file(self.rank))

    def save(self, path, *, step: int, dataloader_state=None, eval_dataloader_state=None, metadata=None) -> None:
        """Write an exact-resume checkpoint of this topology (collective)."""
        self.plane.fence(self.device)
        target = Path(path)

        def make_staging():
            if target.exists():
                raise FileExistsError(f"Checkpoint already exists: {target}")
            target.parent.mkdir(parents=True, exist_ok=True)
            staging = target.with_name(f".{target.name}.partial-{uuid.uuid4().hex}")
            staging.mkdir()
            return str(staging)

        staging = Path(self.plane.on_root("directory setup", make_staging))
        discard = lambda: shutil.rmtree(staging, ignore_errors=True)  # noqa: E731
        self.plane.on_every_rank(
            "write", lambda: self._write_my_files(staging, dataloader_state, eval_dataloader_state), cleanup=discard)

        def publish():
            manifest = {key: compute(self) for key, compute, _ in _MANIFEST_SCHEMA}
            manifest.update(step=int(step), config=self._resolved_config(), metadata=json_safe(metadata or {}))
            try:
                (staging / "manifest.json").write_text(json.dumps(manifest, indent=2, sort_keys=True) + "\n",
                                                       encoding="utf-8")
                (staging / "COMPLETE").write_text("complete\n", encoding="utf-8")
                os.replace(staging, target)
            except BaseException:
                discard()
                raise

        self.plane.on_root("publish", publish)

    def _read_manifest(self, root: Path) -> dict:
        def read():
            if not (root / "COMPLETE").is_file():
                raise FileNotFoundError(f"{root} has no COMPLETE marker (an interrupted or foreign write)")
            return json.loads((root / "manifest.json").read_text(encoding="utf-8"))

        return self.plane.on_root("manifest read", read)

    def load(self, path, *, strict: bool = True) -> dict:
        """Restore model, optimizer, scaler, scheduler, RNG and data position
        from a checkpoint of the same topology (collective)."""
        root = Path(path)
        manifest = self._read_manifest(root)
        for key, compute, problem in _MANIFEST_SCHEMA:  # identical on every rank
            current = compute(self)
            if manifest.get(key) != current:
                raise CheckpointError(problem.format(saved=manifest.get(key), current=current))
        scaler, scheduler = self._engine_extras()

        def restore():
            shard = torch.load(root / self._my_model_file(), map_location="cpu", weights_only=False)
            if shard.get("format_version") != CHECKPOINT_FORMAT_VERSION:
                raise ValueError(f"model shard format_version {shard.get('format_version')!r} is not supported")
            state = torch.load(root / DirectoryLayout.rank_file(self.rank), map_location="cpu", weights_only=False)
            _check_rank_state(state, self.rank, self.device, scaler is not None, scheduler is not None)
            self.load_sharded_state_dict(shard["model"], strict=strict)
            self.engine.optimizer.load_state_dict(shard["optimizer"])
            if scaler is not None:
                scaler.load_state_dict(state["grad_scaler"])
            if scheduler is not None:
                scheduler.load_state_dict(state["scheduler"])
            return state

        state = self.plane.on_every_rank("load", restore)
        # generators last, so nothing above consumes the restored streams
        for name, (_, put) in _rng_sources(self.device).items():
            if name in state["rng"]:
                put(state["rng"][name])
        return {"step": manifest["step"], "dataloader_state": state.get("dataloader"),
                "eval_dataloader_state": state.get("eval_dataloader"),
                "metadata": manifest.get("metadata", {}), "config": manifest.get("config")}
