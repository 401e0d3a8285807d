from .qwen3 import build_qwen3_plan
from .qwen3_moe import build_qwen3_moe_plan

__all__ = ["build_qwen3_plan", "build_qwen3_moe_plan"]
