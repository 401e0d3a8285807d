"""Weights & Biases tracker on rank 0 (no-op elsewhere or when wandb is absent).

Reference: parallel/parallel/tracking.py (asserts WANDB_API_KEY when enabled).
"""
from __future__ import annotations

import os


class WandBTracker:
    def __init__(self, rank: int = 0, project: str | None = None, enabled: bool | None = None):
        self.rank = rank
        self.project = project or os.environ.get("WANDB_PROJECT", "parallel-b200")
        self.enabled = (rank == 0) if enabled is None else (enabled and rank == 0)
        self._run = None
        self._wandb = None

    def start(self):
        if not self.enabled:
            return
        try:
            import wandb  # noqa: F401
        except ImportError:
            self.enabled = False
            return
        assert os.environ.get("WANDB_API_KEY"), "WANDB_API_KEY must be set to track with wandb"
        self._wandb = wandb
        self._run = wandb.init(project=self.project)

    def store_init_config(self, config: dict):
        if self._run is not None:
            self._run.config.update(config)

    def log(self, metrics: dict, step: int | None = None):
        if self._run is not None:
            self._run.log(metrics, step=step)

    def finish(self):
        if self._run is not None:
            self._run.finish()
            self._run = None
