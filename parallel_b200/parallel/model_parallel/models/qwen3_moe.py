"""Qwen3-MoE model-parallel plan (reference: .../model_parallel/models/qwen3_moe.py)."""
from __future__ import annotations

from ..plan import (GradientReduction, ModelParallelCapabilities, ModelParallelPlan, ModuleRule,
                    ParameterParallelism, ParameterPlacement)
from ..registry import register_model_parallel_plan
from .common import qwen_attention_placements, qwen_replicated_placements, require_divisible


@register_model_parallel_plan("qwen3_moe")
def build_qwen3_moe_plan(config, pconfig) -> ModelParallelPlan:
    tp, ep, etp = pconfig.tp_size, pconfig.ep_size, pconfig.expert_tp_size
    sp = getattr(pconfig, "sp_size", 1)
    if tp <= 1 or ep <= 1:
        raise ValueError("Qwen3-MoE folded model parallelism requires tp > 1 and ep > 1")
    if tp != ep:
        raise ValueError("Qwen3-MoE folded model parallelism requires tp == ep")
    if etp != 1:
        raise NotImplementedError("Qwen3-MoE expert tensor parallelism must be 1")
    if sp not in (1, tp):
        raise ValueError("Qwen3-MoE sequence parallelism requires sp == 1 or sp == tp")
    seq = sp > 1
    require_divisible("Qwen3-MoE", "attention heads", config.num_attention_heads, tp)
    require_divisible("Qwen3-MoE", "key/value heads", config.num_key_value_heads, tp)
    require_divisible("Qwen3-MoE", "experts", config.num_experts, ep)
    require_divisible("Qwen3-MoE", "vocabulary size", config.vocab_size, tp)
    col = "colwise_sequence" if seq else "colwise"
    row = "rowwise_sequence" if seq else "rowwise"
    rules = (
        ModuleRule("model.embed_tokens", "embedding_rowwise"),
        ModuleRule("model.layers.*.self_attn.q_proj", col),
        ModuleRule("model.layers.*.self_attn.k_proj", col),
        ModuleRule("model.layers.*.self_attn.v_proj", col),
        ModuleRule("model.layers.*.self_attn.o_proj", row),
        ModuleRule("model.layers.*.mlp.experts.gate_up_proj", "grouped_gemm"),
        ModuleRule("model.layers.*.mlp.experts.down_proj", "grouped_gemm"),
        ModuleRule("lm_head", col),
    )
    P = ParameterParallelism
    red = GradientReduction.SUM_TP if seq else GradientReduction.NONE
    placements = (qwen_attention_placements() + (
        ParameterPlacement("model.layers.*.mlp.gate.weight", P.REPLICATED, gradient_reduction=red),
        ParameterPlacement("model.layers.*.mlp.experts.gate_up_proj", P.EXPERT, 0),
        ParameterPlacement("model.layers.*.mlp.experts.down_proj", P.EXPERT, 0),
    ) + qwen_replicated_placements(seq))
    return ModelParallelPlan(model_type=config.model_type, tensor_parallel_size=tp, expert_parallel_size=ep,
                             expert_tensor_parallel_size=etp, sequence_parallel_size=sp, module_rules=rules,
                             parameter_placements=placements,
                             capabilities=ModelParallelCapabilities(expert_parallel=True, sequence_parallel=seq,
                                                                    fsdp_composition=True))
