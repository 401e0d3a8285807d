"""Barrier helper (reference: parallel/parallel/collectives.py)."""
from __future__ import annotations

import torch
import torch.distributed as dist


def wait_for_everyone() -> None:
    """Barrier across all ranks; on NCCL also drains the current device."""
    if not (dist.is_available() and dist.is_initialized()):
        return
    if dist.get_backend() == "nccl" and torch.cuda.is_available():
        dist.barrier(device_ids=[torch.cuda.current_device()])
    else:
        dist.barrier()
