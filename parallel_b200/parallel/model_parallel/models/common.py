"""Shared construction of the Qwen3 / Qwen3-MoE model-parallel plans.

The placement table (patterns, their order, placements, shard dims, required
flags and gradient reductions) is recorded in model-parallel checkpoints and
compared on load, so it must equal the reference's table
(``parallel/parallel/engine/model_parallel/models/{common,qwen3,qwen3_moe}.py``)
entry for entry.  It is written here as compact rows:
``(pattern, parallelism, shard_dim, required, reduction)`` where
``reduction`` is ``"sum"`` (always summed over TP), ``"sp"`` (summed over TP
only under sequence parallelism) or ``None``.

``build_qwen_plan`` turns a family description (name, MLP rows, module
roles, the config sizes that must divide by TP) into a ``ModelParallelPlan``.
"""
from __future__ import annotations

from dataclasses import dataclass

from ..plan import (GradientReduction, ModelParallelCapabilities, ModelParallelPlan, ModuleRule,
                    ParameterParallelism, ParameterPlacement)

_L = "model.layers.*."

# attention block + embedding / LM head, in table order
ATTENTION_ROWS = (
    ("model.embed_tokens.weight", "vocab", 0, True, None),
    (_L + "self_attn.q_proj.weight", "column", 0, True, None),
    (_L + "self_attn.q_proj.bias", "column", 0, False, None),
    (_L + "self_attn.k_proj.weight", "column", 0, True, None),
    (_L + "self_attn.k_proj.bias", "column", 0, False, None),
    (_L + "self_attn.v_proj.weight", "column", 0, True, None),
    (_L + "self_attn.v_proj.bias", "column", 0, False, None),
    (_L + "self_attn.q_norm.weight", "replicated", None, True, "sum"),
    (_L + "self_attn.k_norm.weight", "replicated", None, True, "sum"),
    (_L + "self_attn.o_proj.weight", "row", 1, True, None),
    (_L + "self_attn.o_proj.bias", "replicated", None, False, None),
    ("lm_head.weight", "vocab", 0, False, None),
)
# norms (replicated; their gradients are partial per rank only under SP)
NORM_ROWS = (
    (_L + "input_layernorm.weight", "replicated", None, True, "sp"),
    (_L + "post_attention_layernorm.weight", "replicated", None, True, "sp"),
    ("model.norm.weight", "replicated", None, True, "sp"),
)
# module -> role; the role picks the HF TP style
ATTENTION_MODULES = (("model.embed_tokens", "embedding"), (_L + "self_attn.q_proj", "col"),
                     (_L + "self_attn.k_proj", "col"), (_L + "self_attn.v_proj", "col"),
                     (_L + "self_attn.o_proj", "row"))


def _style(role: str, sequence_parallel: bool) -> str:
    base = {"col": "colwise", "row": "rowwise", "embedding": "embedding_rowwise", "grouped": "grouped_gemm"}[role]
    return base + "_sequence" if sequence_parallel and role in ("col", "row") else base


def placements_from_rows(rows, sequence_parallel: bool) -> tuple[ParameterPlacement, ...]:
    def reduction(tag):
        summed = tag == "sum" or (tag == "sp" and sequence_parallel)
        return GradientReduction.SUM_TP if summed else GradientReduction.NONE

    return tuple(ParameterPlacement(pattern, ParameterParallelism(kind), dim, required, reduction(tag))
                 for pattern, kind, dim, required, tag in rows)


def require_divisible(model_name: str, name: str, value: int, divisor: int) -> None:
    if value % divisor:
        raise ValueError(f"{model_name}: {name} = {value} is not divisible by the TP size {divisor}")


@dataclass(frozen=True)
class QwenFamily:
    label: str                      # for messages
    expert_parallel: bool
    mlp_rows: tuple                 # placement rows of the MLP block
    mlp_modules: tuple              # (module pattern, role) of the MLP block
    divisible: tuple                # (config attribute, description) that TP must divide


def build_qwen_plan(config, pconfig, family: QwenFamily) -> ModelParallelPlan:
    tp, ep, etp = pconfig.tp_size, pconfig.ep_size, pconfig.expert_tp_size
    sp = getattr(pconfig, "sp_size", 1)
    name = family.label
    if family.expert_parallel:
        problems = [(tp <= 1 or ep <= 1, ValueError, f"{name} model parallelism folds EP onto TP and needs "
                                                     f"tp > 1 and ep > 1 (tp={tp}, ep={ep})"),
                    (tp != ep, ValueError, f"{name} runs experts on the TP ranks: tp == ep is required"),
                    (etp != 1, NotImplementedError, f"{name}: expert_tp must be 1")]
    else:
        problems = [(tp <= 1, ValueError, f"{name} tensor parallelism needs tp > 1 (tp={tp})"),
                    (ep != 1, ValueError, f"{name} is dense: ep must be 1"),
                    (etp != 1, ValueError, f"{name} is dense: expert_tp must be 1")]
    problems.append((sp not in (1, tp), ValueError, f"{name}: sp must be 1 or equal to tp (sp == 1 or sp == tp)"))
    for failed, kind, message in problems:
        if failed:
            raise kind(message)
    for attr, what in family.divisible:
        require_divisible(name, what, getattr(config, attr), tp)
    seq = sp > 1
    modules = ATTENTION_MODULES + family.mlp_modules + (("lm_head", "col"),)
    rows = ATTENTION_ROWS + family.mlp_rows + NORM_ROWS
    return ModelParallelPlan(
        model_type=config.model_type, tensor_parallel_size=tp, expert_parallel_size=ep if family.expert_parallel else 1,
        expert_tensor_parallel_size=etp if family.expert_parallel else 1, sequence_parallel_size=sp,
        module_rules=tuple(ModuleRule(pattern, _style(role, seq)) for pattern, role in modules),
        parameter_placements=placements_from_rows(rows, seq),
        capabilities=ModelParallelCapabilities(expert_parallel=family.expert_parallel, sequence_parallel=seq,
                                               fsdp_composition=True))
