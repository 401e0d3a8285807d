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
import re
from dataclasses import dataclass, field, fields
from enum import Enum
from functools import lru_cache
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
        return _pattern(self.pattern).match(name) is not None


@dataclass(frozen=True)
class ModelParallelCapabilities:
    tensor_parallel: bool = True
    expert_parallel: bool = False
    expert_tensor_parallel: bool = False
    sequence_parallel: bool = False
    fsdp_composition: bool = False
    portable_checkpoint: bool = True
    sharded_checkpoint: bool = True


# checkpoint_metadata() records these plan fields, in this order, then the placements
_METADATA_FIELDS = ("model_type", "tensor_parallel_size", "expert_parallel_size", "expert_tensor_parallel_size",
                    "sequence_parallel_size")


def _plain(value):
    return value.value if isinstance(value, Enum) else value


@lru_cache(maxsize=None)
def _pattern(glob: str) -> "re.Pattern":
    return re.compile(fnmatch.translate(glob))


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
        return dict((rule.pattern, rule.style) for rule in self.module_rules)

    def _first_match(self, name: str):
        """Index of the first placement whose pattern matches ``name`` (the
        table is ordered most-specific first), or None."""
        cache = self.__dict__.setdefault("_match_cache", {})
        if name not in cache:
            cache[name] = next((i for i, pl in enumerate(self.parameter_placements)
                                if _pattern(pl.pattern).match(name)), None)
        return cache[name]

    def placement_for_parameter(self, name: str) -> ParameterPlacement:
        index = self._first_match(name)
        if index is None:
            raise KeyError(f"no placement of the {self.model_type} plan matches parameter {name!r}")
        return self.parameter_placements[index]

    def validate_parameter_coverage(self, names: Iterable[str]) -> None:
        """Every parameter must have a placement, and every required placement
        must match at least one parameter."""
        names = list(names)
        orphans = [n for n in names if self._first_match(n) is None]
        if orphans:
            raise RuntimeError(f"the {self.model_type} plan has no placement for: {', '.join(orphans)}")
        unmatched = [pl.pattern for pl in self.parameter_placements
                     if pl.required and not any(_pattern(pl.pattern).match(n) for n in names)]
        if unmatched:
            raise RuntimeError(f"the model has no parameter for required plan entries: {', '.join(unmatched)}")

    def checkpoint_metadata(self) -> dict:
        """Plan description stored with model-parallel checkpoints and compared
        for equality when they are loaded (an interchange format)."""
        meta = {key: getattr(self, key) for key in _METADATA_FIELDS}
        meta["parameters"] = [{f.name: _plain(getattr(pl, f.name)) for f in fields(ParameterPlacement)}
                              for pl in self.parameter_placements]
        return meta

    def validate_runtime(self, pconfig) -> None:
        checks = (
            (self.sequence_parallel_size not in (1, self.tensor_parallel_size), ValueError,
             f"sequence parallel size {self.sequence_parallel_size} must be 1 or the TP size "
             f"{self.tensor_parallel_size}"),
            (pconfig.dp_shard_size > 1 and not self.capabilities.fsdp_composition, NotImplementedError,
             f"the {self.model_type} plan does not compose with FSDP; use dp_shard=1"),
            (self.expert_tensor_parallel_size > 1 and not self.capabilities.expert_tensor_parallel,
             NotImplementedError, f"the {self.model_type} plan has no expert tensor parallelism"),
        )
        for failed, kind, message in checks:
            if failed:
                raise kind(message)
