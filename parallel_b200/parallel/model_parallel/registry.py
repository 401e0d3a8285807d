"""Registry of plan builders keyed by ``config.model_type``
(reference: parallel/parallel/engine/model_parallel/registry.py)."""
from __future__ import annotations

from collections.abc import Callable

from .plan import ModelParallelPlan

PlanBuilder = Callable[[object, object], ModelParallelPlan]
_BUILDERS: dict[str, PlanBuilder] = {}


def register_model_parallel_plan(model_type: str):
    def deco(builder: PlanBuilder) -> PlanBuilder:
        if model_type in _BUILDERS:
            raise RuntimeError(f"Duplicate model-parallel plan for {model_type}")
        _BUILDERS[model_type] = builder
        return builder

    return deco


def build_model_parallel_plan(config, pconfig) -> ModelParallelPlan:
    mt = getattr(config, "model_type", None)
    builder = _BUILDERS.get(mt)
    if builder is None:
        raise NotImplementedError(f"Model parallelism does not support model_type={mt!r}; supported model types: "
                                  + ", ".join(sorted(_BUILDERS)))
    return builder(config, pconfig)


def supported_model_types() -> tuple[str, ...]:
    return tuple(sorted(_BUILDERS))
