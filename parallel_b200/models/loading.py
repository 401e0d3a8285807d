"""Model construction / loading (reference: parallel/parallel/engine/model_loading.py).

``load_causal_lm(cfg, pconfig)`` returns ``(model, plan_or_None)``:
* no model parallelism: the full model (bf16, HF init or weights from a
  local directory), placed on the device later by FSDP / the trainer;
* model parallelism: the plan is built from the registry and validated, and
  every rank materialises only its local shards.

``model.name`` is a local HF-style directory (``config.json`` plus
``model.safetensors`` / ``pytorch_model.bin`` / ``model.pt``) or one of the
preset architecture names in ``models/config.py`` (random-init weights; no
network access is needed or attempted).
"""
from __future__ import annotations

import glob
import os
from collections import OrderedDict

import torch

from .config import ModelConfig, resolve_config
from .qwen3 import Qwen3ForCausalLM, build_model


def read_state_dict(path: str):
    """Full state dict from a local directory (None when it has no weights)."""
    st = sorted(glob.glob(os.path.join(path, "*.safetensors")))
    if st:
        try:
            from safetensors.torch import load_file
        except ImportError as exc:  # pragma: no cover
            raise RuntimeError("safetensors is required to read *.safetensors weights") from exc
        out = OrderedDict()
        for f in st:
            out.update(load_file(f))
        return out
    for name in ("pytorch_model.bin", "model.pt"):
        f = os.path.join(path, name)
        if os.path.exists(f):
            return torch.load(f, map_location="cpu", weights_only=False)
    return None


def save_pretrained(model: Qwen3ForCausalLM, path: str) -> None:
    """config.json + model.pt (a portable state dict)."""
    os.makedirs(path, exist_ok=True)
    model.config.save_pretrained(path)
    sd = OrderedDict((k, v.detach().cpu()) for k, v in model.state_dict().items())
    torch.save(sd, os.path.join(path, "model.pt"))


def _model_config(cfg) -> ModelConfig:
    mcfg = resolve_config(cfg.model.name)
    if mcfg.is_moe:
        mcfg.output_router_logits = bool(cfg.model.get("output_router_logits", True))
    return mcfg


def load_causal_lm(cfg, pconfig, dtype=torch.bfloat16, seed: int | None = None):
    config = _model_config(cfg)
    if not pconfig.model_parallel_enabled:
        model = build_model(config, dtype=dtype, seed=seed)
        if os.path.isdir(cfg.model.name):
            sd = read_state_dict(cfg.model.name)
            if sd is not None:
                model.load_state_dict(sd, strict=False)
                model._layout_fused_weights()
        return model, None
    from ..parallel.model_parallel import build_model_parallel_plan
    from ..parallel.model_parallel.tensor_parallel import load_tensor_parallel_causal_lm

    plan = build_model_parallel_plan(config, pconfig)
    plan.validate_runtime(pconfig)
    model = load_tensor_parallel_causal_lm(cfg.model.name, config=config, pconfig=pconfig, plan=plan, dtype=dtype,
                                           seed=seed)
    return model, plan
