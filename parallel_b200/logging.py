"""Rank-aware logging: rank 0 by default, or every rank in rank order.

Level from ``PARALLEL_LOG_LEVEL`` (reference: parallel/parallel/logging.py).
"""
from __future__ import annotations

import logging
import os

import torch.distributed as dist


def configure_logging(level: str | None = None) -> None:
    level = (level or os.environ.get("PARALLEL_LOG_LEVEL", "INFO")).upper()
    logging.basicConfig(level=getattr(logging, level, logging.INFO),
                        format="%(asctime)s %(levelname)s %(name)s: %(message)s", force=True)


def _rank_world():
    if dist.is_available() and dist.is_initialized():
        return dist.get_rank(), dist.get_world_size()
    return int(os.environ.get("RANK", 0)), int(os.environ.get("WORLD_SIZE", 1))


class MultiProcAdapter(logging.LoggerAdapter):
    """``main_process_only=True`` (default) logs on rank 0; ``in_order=True``
    logs on every rank, one rank at a time (barrier between ranks)."""

    def log(self, level, msg, *args, main_process_only: bool = True, in_order: bool = False, **kwargs):
        if not self.isEnabledFor(level):
            return
        rank, world = _rank_world()
        if in_order and world > 1 and dist.is_initialized():
            for r in range(world):
                if r == rank:
                    msg2, kw = self.process(msg, kwargs)
                    self.logger.log(level, msg2, *args, **kw)
                dist.barrier()
            return
        if main_process_only and rank != 0:
            return
        msg2, kw = self.process(msg, kwargs)
        self.logger.log(level, msg2, *args, **kw)

    def process(self, msg, kwargs):
        rank, _ = _rank_world()
        return f"[rank{rank}] {msg}", kwargs


def get_logger(name: str, level: str | None = None) -> MultiProcAdapter:
    logger = logging.getLogger(name)
    if level is not None:
        logger.setLevel(level.upper())
    return MultiProcAdapter(logger, {})
