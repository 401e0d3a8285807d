"""Small shared helpers (dtype table, distributed-state predicates, env patching)."""
from __future__ import annotations

import os
from contextlib import contextmanager

import torch
import torch.distributed as dist

DTYPE_DICT = {
    "bf16": torch.bfloat16,
    "fp16": torch.float16,
}


def empty_fn(*args, **kwargs):
    pass


@contextmanager
def patch_environment(**kwargs):
    """Temporarily set upper-cased environment variables."""
    saved = {}
    for key, value in kwargs.items():
        key = key.upper()
        if key in os.environ:
            saved[key] = os.environ[key]
        os.environ[key] = str(value)
    try:
        yield
    finally:
        for key in kwargs:
            key = key.upper()
            if key in saved:
                os.environ[key] = saved[key]
            else:
                os.environ.pop(key, None)


def is_cuda_available() -> bool:
    with patch_environment(PYTORCH_NVML_BASED_CUDA_CHECK="1"):
        return torch.cuda.is_available()


def is_dist_initialized() -> bool:
    return dist.is_available() and dist.is_initialized()


def dist_cleanup() -> None:
    if is_dist_initialized():
        dist.barrier()
        dist.destroy_process_group()
