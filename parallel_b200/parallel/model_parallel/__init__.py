from . import models as models
from .api import ModelParallelWrapper
from .expert_parallel import ExpertPartition, ReplicatedTokenExpertParallel, SequenceParallelExpertParallel
from .models import build_qwen3_moe_plan, build_qwen3_plan
from .plan import (GradientReduction, ModelParallelCapabilities, ModelParallelPlan, ModuleRule,
                   ParameterParallelism, ParameterPlacement)
from .registry import build_model_parallel_plan, supported_model_types
from .sequence_parallel import SequenceParallelRuntime
from .token_dispatch import TokenDispatcher

__all__ = [
    "ExpertPartition", "GradientReduction", "ModelParallelCapabilities", "ModelParallelPlan",
    "ModelParallelWrapper", "ModuleRule", "ParameterParallelism", "ParameterPlacement",
    "ReplicatedTokenExpertParallel", "SequenceParallelExpertParallel", "SequenceParallelRuntime",
    "TokenDispatcher", "build_model_parallel_plan", "build_qwen3_moe_plan", "build_qwen3_plan",
    "supported_model_types",
]
