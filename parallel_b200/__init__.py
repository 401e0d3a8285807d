"""parallel_b200: a Blackwell-native composable-parallelism training engine for Qwen3 / Qwen3-MoE.

Public entry points mirror ``jonahsamost/parallel``: ``profile`` (timing
helper), the training CLI (``python -m parallel_b200.train key=value ...``),
``parallel_b200.parallel.engine.ParallelEngine`` and friends.
"""
from .profiling import profile

__all__ = ["profile"]
__version__ = "0.1.0"
