"""Loader for the in-tree sm_100a extension (``parallel_b200/_C*.so``).

On a machine with a CUDA device the extension is mandatory: a missing or
stale build raises immediately instead of silently running PyTorch eager
code.  On a CPU-only machine every op runs its fp32/bf16 PyTorch
restatement (the numerics oracle used by the CPU test-suite).
"""
from __future__ import annotations

import importlib

import torch

_C = None
_err: Exception | None = None
try:
    _C = importlib.import_module("parallel_b200._C")
except Exception as exc:  # pragma: no cover - depends on the build
    _err = exc


_resolved = None


def ext():
    """Return the compiled module, raising loudly if it is unavailable.  With
    ``PB_COMM_DEBUG=1`` (read once per process) the peer-memory launches go
    through the span and guard-word checks of ``parallel_b200.parallel.comm.debug``."""
    global _resolved
    if _resolved is not None:
        return _resolved
    if _C is None:
        raise RuntimeError(
            "parallel_b200._C (sm_100a kernels) is not built or failed to load: "
            f"{_err!r}. Build it with `python setup.py build_ext --inplace`."
        )
    from ..parallel.comm import debug

    _resolved = debug.checked_extension(_C) if debug.enabled() else _C
    return _resolved


def available() -> bool:
    return _C is not None


def use_kernels(t: torch.Tensor) -> bool:
    """True when ``t`` lives on a CUDA device, i.e. the native kernels must run."""
    if t.is_cuda:
        ext()
        return True
    return False


def clear_device_errors(device: int | None = None) -> None:
    if _C is not None:
        _C.clear_error(torch.cuda.current_device() if device is None else device)


def check_device_errors(device: int | None = None) -> None:
    """Raise if any kernel on ``device`` recorded a bounded-wait timeout."""
    if _C is None:
        return
    dev = torch.cuda.current_device() if device is None else device
    code = _C.read_error(dev)
    if code:
        _C.clear_error(dev)
        raise RuntimeError(f"parallel_b200 kernel reported error code {code} on cuda:{dev} "
                           "(1 = pipeline wait timeout, 2 = peer wait timeout, 3 = bad argument, "
                           "4 = MoE layout over capacity, 5 = split-K slice wait timeout)")
