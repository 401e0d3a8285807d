"""Qwen3-MoE: attention as dense Qwen3; whole experts owned by TP ranks (EP
folded onto TP), router replicated (behaviour of
``parallel/parallel/engine/model_parallel/models/qwen3_moe.py``)."""
from __future__ import annotations

from ..plan import ModelParallelPlan
from ..registry import register_model_parallel_plan
from .common import _L, QwenFamily, build_qwen_plan

QWEN3_MOE = QwenFamily(
    label="Qwen3-MoE",
    expert_parallel=True,
    mlp_rows=((_L + "mlp.gate.weight", "replicated", None, True, "sp"),
              (_L + "mlp.experts.gate_up_proj", "expert", 0, True, None),
              (_L + "mlp.experts.down_proj", "expert", 0, True, None)),
    mlp_modules=((_L + "mlp.experts.gate_up_proj", "grouped"), (_L + "mlp.experts.down_proj", "grouped")),
    divisible=(("num_attention_heads", "attention heads"), ("num_key_value_heads", "key/value heads"),
               ("num_experts", "experts"), ("vocab_size", "vocabulary size")),
)


@register_model_parallel_plan("qwen3_moe")
def build_qwen3_moe_plan(config, pconfig) -> ModelParallelPlan:
    return build_qwen_plan(config, pconfig, QWEN3_MOE)
