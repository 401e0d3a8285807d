"""Small shared helpers: the config-string -> torch dtype table and the
process-group lifetime predicates used by the state and the training CLI
(the reference keeps the same names in ``parallel/utils.py``)."""
from __future__ import annotations

import torch
import torch.distributed as dist

# config strings accepted by ``engine.dtype`` style keys
DTYPE_DICT = {"bf16": torch.bfloat16, "fp16": torch.float16}


def is_dist_initialized() -> bool:
    """True once a default process group exists (False on builds without
    torch.distributed)."""
    return bool(dist.is_available() and dist.is_initialized())


def dist_cleanup() -> None:
    """Leave the job in step with the other ranks, then tear the default
    process group down; a no-op in single-process runs."""
    if not is_dist_initialized():
        return
    dist.barrier()
    dist.destroy_process_group()
