"""Placement tables shared by the Qwen3 plans.

The pattern/placement table is the checkpoint-metadata contract with the
reference (parallel/parallel/engine/model_parallel/models/common.py), so it
lists the same patterns in the same order.
"""
from __future__ import annotations

from ..plan import GradientReduction, ParameterParallelism, ParameterPlacement


def require_divisible(model_name: str, name: str, value: int, divisor: int) -> None:
    if value % divisor:
        raise ValueError(f"{model_name} {name} ({value}) must be divisible by tensor-parallel size ({divisor})")


def qwen_attention_placements() -> tuple[ParameterPlacement, ...]:
    P, R = ParameterParallelism, GradientReduction
    Pl = ParameterPlacement
    return (
        Pl("model.embed_tokens.weight", P.VOCAB, 0),
        Pl("model.layers.*.self_attn.q_proj.weight", P.COLUMN, 0),
        Pl("model.layers.*.self_attn.q_proj.bias", P.COLUMN, 0, False),
        Pl("model.layers.*.self_attn.k_proj.weight", P.COLUMN, 0),
        Pl("model.layers.*.self_attn.k_proj.bias", P.COLUMN, 0, False),
        Pl("model.layers.*.self_attn.v_proj.weight", P.COLUMN, 0),
        Pl("model.layers.*.self_attn.v_proj.bias", P.COLUMN, 0, False),
        Pl("model.layers.*.self_attn.q_norm.weight", P.REPLICATED, gradient_reduction=R.SUM_TP),
        Pl("model.layers.*.self_attn.k_norm.weight", P.REPLICATED, gradient_reduction=R.SUM_TP),
        Pl("model.layers.*.self_attn.o_proj.weight", P.ROW, 1),
        Pl("model.layers.*.self_attn.o_proj.bias", P.REPLICATED, None, False),
        Pl("lm_head.weight", P.VOCAB, 0, False),
    )


def qwen_replicated_placements(sequence_parallel: bool = False) -> tuple[ParameterPlacement, ...]:
    P = ParameterParallelism
    red = GradientReduction.SUM_TP if sequence_parallel else GradientReduction.NONE
    Pl = ParameterPlacement
    return (
        Pl("model.layers.*.input_layernorm.weight", P.REPLICATED, gradient_reduction=red),
        Pl("model.layers.*.post_attention_layernorm.weight", P.REPLICATED, gradient_reduction=red),
        Pl("model.norm.weight", P.REPLICATED, gradient_reduction=red),
    )
