"""Lookup of model-parallel plan builders by HF ``config.model_type``.

Plan modules declare themselves with ``@register_model_parallel_plan(type)``
(behaviour of ``parallel/parallel/engine/model_parallel/registry.py``).  A
builder is ``(model_config, pconfig) -> ModelParallelPlan``.
"""
from __future__ import annotations

from collections.abc import Callable
from types import MappingProxyType

from .plan import ModelParallelPlan

PlanBuilder = Callable[[object, object], ModelParallelPlan]


class _PlanTable:
    def __init__(self):
        self._builders: dict[str, PlanBuilder] = {}
        self.view = MappingProxyType(self._builders)

    def add(self, model_type: str, builder: PlanBuilder) -> None:
        previous = self._builders.get(model_type)
        if previous is not None and previous is not builder:
            raise RuntimeError(f"model_type {model_type!r} already has a plan builder ({previous.__qualname__})")
        self._builders[model_type] = builder


_TABLE = _PlanTable()


def register_model_parallel_plan(model_type: str):
    """Decorator: make ``builder`` the plan of ``model_type``."""
    def bind(builder: PlanBuilder) -> PlanBuilder:
        _TABLE.add(model_type, builder)
        return builder

    return bind


def supported_model_types() -> tuple[str, ...]:
    return tuple(sorted(_TABLE.view))


def build_model_parallel_plan(config, pconfig) -> ModelParallelPlan:
    model_type = getattr(config, "model_type", None)
    if model_type not in _TABLE.view:
        raise NotImplementedError(f"no model-parallel plan for model_type {model_type!r} "
                                  f"(plans exist for: {', '.join(supported_model_types()) or 'none'})")
    return _TABLE.view[model_type](config, pconfig)
