"""Dense Qwen3: attention heads, KV heads and the MLP split column / row over TP
(behaviour of ``parallel/parallel/engine/model_parallel/models/qwen3.py``)."""
from __future__ import annotations

from ..plan import ModelParallelPlan
from ..registry import register_model_parallel_plan
from .common import _L, QwenFamily, build_qwen_plan

QWEN3 = QwenFamily(
    label="Qwen3",
    expert_parallel=False,
    mlp_rows=((_L + "mlp.gate_proj.weight", "column", 0, True, None),
              (_L + "mlp.up_proj.weight", "column", 0, True, None),
              (_L + "mlp.down_proj.weight", "row", 1, True, None)),
    mlp_modules=((_L + "mlp.gate_proj", "col"), (_L + "mlp.up_proj", "col"), (_L + "mlp.down_proj", "row")),
    divisible=(("num_attention_heads", "attention heads"), ("num_key_value_heads", "key/value heads"),
               ("intermediate_size", "intermediate size"), ("vocab_size", "vocabulary size")),
)


@register_model_parallel_plan("qwen3")
def build_qwen3_plan(config, pconfig) -> ModelParallelPlan:
    return build_qwen_plan(config, pconfig, QWEN3)
