"""Configuration: YAML defaults + optional override YAML + ``a.b=c`` overrides.

Same merge semantics as the reference's OmegaConf-based loader
(parallel/parallel/utils.py:20-40): the first ``*.yaml`` argument is merged
over ``conf/default.yaml``, then every ``key.path=value`` argument is merged
in order.  Values are parsed as YAML scalars (ints, floats incl. ``1e-5``,
booleans, ``null``), so ``parallel.tp=2`` is an int and ``engine.activation_
checkpoint=true`` a bool.  Nodes support attribute and item access and
``.get``; ``to_container`` returns plain dicts.
"""
from __future__ import annotations

import copy
import re
import sys
from pathlib import Path
from typing import Any, Iterable

import yaml

_FLOAT_RE = re.compile(r"^[-+]?(\d+\.?\d*|\.\d+)([eE][-+]?\d+)?$")


class Config(dict):
    """A dict with attribute access; nested dicts become Config nodes."""

    def __init__(self, data: dict | None = None):
        super().__init__()
        for k, v in (data or {}).items():
            self[k] = v

    def __setitem__(self, key, value):
        if isinstance(value, dict) and not isinstance(value, Config):
            value = Config(value)
        super().__setitem__(key, value)

    def __getattr__(self, key):
        try:
            return self[key]
        except KeyError as exc:
            raise AttributeError(key) from exc

    def __setattr__(self, key, value):
        self[key] = value

    def __delattr__(self, key):
        del self[key]

    def __deepcopy__(self, memo):
        return Config(copy.deepcopy(dict(self), memo))

    def to_container(self) -> dict:
        return {k: (v.to_container() if isinstance(v, Config) else copy.deepcopy(v)) for k, v in self.items()}

    def select(self, dotted: str, default: Any = None) -> Any:
        node: Any = self
        for part in dotted.split("."):
            if not isinstance(node, dict) or part not in node:
                return default
            node = node[part]
        return node


def parse_scalar(text: str) -> Any:
    """YAML-1.2-like scalar parsing (``1e-5`` is a float, unlike PyYAML)."""
    t = text.strip()
    if _FLOAT_RE.match(t) and not re.match(r"^[-+]?\d+$", t):
        return float(t)
    try:
        v = yaml.safe_load(t)
    except yaml.YAMLError:
        return t
    return v


def _fix_floats(node: Any) -> Any:
    if isinstance(node, dict):
        return {k: _fix_floats(v) for k, v in node.items()}
    if isinstance(node, list):
        return [_fix_floats(v) for v in node]
    if isinstance(node, str) and _FLOAT_RE.match(node.strip()):
        return parse_scalar(node)
    return node


def load_yaml(path: str | Path) -> Config:
    with open(path) as f:
        data = yaml.safe_load(f) or {}
    if not isinstance(data, dict):
        raise ValueError(f"{path}: top level must be a mapping")
    return Config(_fix_floats(data))


def merge(base: dict, override: dict) -> Config:
    """Recursive merge; override wins; returns a new Config."""
    out = Config(copy.deepcopy(dict(base)))
    for k, v in override.items():
        if isinstance(v, dict) and isinstance(out.get(k), dict):
            out[k] = merge(out[k], v)
        else:
            out[k] = copy.deepcopy(v)
    return out


def from_dotlist(items: Iterable[str]) -> Config:
    out = Config()
    for item in items:
        if "=" not in item:
            raise ValueError(f"override {item!r} is not of the form key=value")
        key, value = item.split("=", 1)
        node = out
        parts = key.strip().split(".")
        for part in parts[:-1]:
            if part not in node or not isinstance(node[part], dict):
                node[part] = Config()
            node = node[part]
        node[parts[-1]] = parse_scalar(value)
    return out


def default_config_path() -> Path:
    return Path(__file__).parent / "conf" / "default.yaml"


def load_cfg(path: str | Path | None = None, argv: list[str] | None = None) -> Config:
    """defaults (or ``path``) <- first *.yaml argument <- dotted overrides."""
    base = load_yaml(path or default_config_path())
    args = sys.argv[1:] if argv is None else argv
    yaml_args = [a for a in args if a.endswith((".yaml", ".yml"))]
    dot = [a for a in args if "=" in a and not a.endswith((".yaml", ".yml"))]
    cfg = merge(base, load_yaml(yaml_args[0])) if yaml_args else base
    if dot:
        cfg = merge(cfg, from_dotlist(dot))
    return cfg


def to_container(cfg: Config) -> dict:
    return cfg.to_container() if isinstance(cfg, Config) else copy.deepcopy(dict(cfg))
