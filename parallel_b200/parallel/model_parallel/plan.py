"""Model-independent model-parallel placement plan.

A plan maps HF module patterns to TP "styles" and every parameter name
(fnmatch pattern) to a placement: replicated / column / row / vocab / expert,
the dimension it is sharded on, whether it must exist, and whether its
gradient is summed over the TP group.  ``checkpoint_metadata()`` is written
into exact-topology checkpoints and compared for equality on load, so the
field names and values are the reference's (parallel/parallel/engine/
model_parallel/plan.py:9-143).
"""
from __future__ import annotations

import fnmatch
from dataclasses import dataclass, field
from enum import Enum
from typing import Iterable


class ParameterParallelism(str, Enum):
    REPLICATED = "replicated"
    COLUMN = "column"
    ROW = "row"
    VOCAB = "vocab"
    EXPERT = "expert"


class GradientReduction(str, Enum):
    NONE = "none"
    SUM_TP = "sum_tp"


@dataclass(frozen=True)
class ModuleRule:
    pattern: str
    style: str


@dataclass(frozen=True)
class ParameterPlacement:
    pattern: str
    parallelism: ParameterParallelism
    shard_dim: int | None = None
    required: bool = True
    gradient_reduction: GradientReduction = GradientReduction.NONE

    def matches(self, name: str) -> bool:
        return fnmatch.fnmatchcase(name, self.pattern)


@dataclass(frozen=True)
class ModelParallelCapabilities:
    tensor_parallel: bool = True
    expert_parallel: bool = False
    expert_tensor_parallel: bool = False
    sequence_parallel: bool = False
    fsdp_composition: bool = False
    portable_checkpoint: bool = True
    sharded_checkpoint: bool = True


@dataclass(frozen=True)
class ModelParallelPlan:
    model_type: str
    tensor_parallel_size: int
    expert_parallel_size: int
    expert_tensor_parallel_size: int
    sequence_parallel_size: int
    module_rules: tuple[ModuleRule, ...]
    parameter_placements: tuple[ParameterPlacement, ...]
    capabilities: ModelParallelCapabilities = field(default_factory=ModelParallelCapabilities)

    @property
    def size(self) -> int:
        return self.tensor_parallel_size

    @property
    def attention_tp_size(self) -> int:
        return self.tensor_parallel_size

    @property
    def hf_plan(self) -> dict[str, str]:
        return {r.pattern: r.style for r in self.module_rules}

    def placement_for_parameter(self, name: str) -> ParameterPlacement:
        for p in self.parameter_placements:
            if p.matches(name):
                return p
        raise KeyError(f"Model-parallel plan does not classify parameter {name!r}")

    def validate_parameter_coverage(self, names: Iterable[str]) -> None:
        names = tuple(names)
        unclassified = []
        for n in names:
            try:
                self.placement_for_parameter(n)
            except KeyError:
                unclassified.append(n)
        if unclassified:
            raise RuntimeError("Model-parallel plan leaves parameters unclassified: " + ", ".join(unclassified))
        missing = [p.pattern for p in self.parameter_placements if p.required and not any(p.matches(n) for n in names)]
        if missing:
            raise RuntimeError("Model-parallel plan expected parameters matching: " + ", ".join(missing))

    def checkpoint_metadata(self) -> dict:
        return {
            "model_type": self.model_type,
            "tensor_parallel_size": self.tensor_parallel_size,
            "expert_parallel_size": self.expert_parallel_size,
            "expert_tensor_parallel_size": self.expert_tensor_parallel_size,
            "sequence_parallel_size": self.sequence_parallel_size,
            "parameters": [
                {"pattern": p.pattern, "parallelism": p.parallelism.value, "shard_dim": p.shard_dim,
                 "required": p.required, "gradient_reduction": p.gradient_reduction.value}
                for p in self.parameter_placements
            ],
        }

    def validate_runtime(self, pconfig) -> None:
        if self.sequence_parallel_size not in (1, self.tensor_parallel_size):
            raise ValueError("Sequence parallelism must be disabled or reuse the complete TP group")
        if pconfig.dp_shard_size > 1 and not self.capabilities.fsdp_composition:
            raise NotImplementedError(f"{self.model_type} model parallelism does not yet compose with FSDP; "
                                      "set dp_shard=1")
        if self.expert_tensor_parallel_size > 1 and not self.capabilities.expert_tensor_parallel:
            raise NotImplementedError(f"{self.model_type} does not support expert tensor parallelism")
