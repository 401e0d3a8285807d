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
import json
import os
from collections import OrderedDict

import torch

from .config import ModelConfig, resolve_config
from .qwen3 import Qwen3ForCausalLM, build_model


def _with_tied_head(path: str, sd):
    """HF checkpoints of tied models store the embedding once: restore the
    ``lm_head.weight`` alias when the config ties them."""
    if sd is None or "lm_head.weight" in sd or "model.embed_tokens.weight" not in sd:
        return sd
    tie = True
    cfg_path = os.path.join(path, "config.json")
    if os.path.exists(cfg_path):
        with open(cfg_path) as f:
            tie = bool(json.load(f).get("tie_word_embeddings", True))
    if tie:
        sd["lm_head.weight"] = sd["model.embed_tokens.weight"]
    return sd


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
        return _with_tied_head(path, out)
    for name in ("pytorch_model.bin", "model.pt"):
        f = os.path.join(path, name)
        if os.path.exists(f):
            return _with_tied_head(path, torch.load(f, map_location="cpu", weights_only=False))
    return None


def save_pretrained(model: Qwen3ForCausalLM, path: str) -> None:
    """config.json + model.safetensors in the Hugging Face layout (a tied LM
    head is stored once, as HF does), loadable by ``transformers`` and by the
    reference's model loading; model.pt when safetensors is unavailable."""
    os.makedirs(path, exist_ok=True)
    model.config.save_pretrained(path)
    # record the dtype the weights are stored in, so loaders that follow the
    # config's dtype (HF "auto") keep them exact
    dtype = next(model.parameters()).dtype
    name = {torch.float32: "float32", torch.bfloat16: "bfloat16", torch.float16: "float16"}.get(dtype)
    if name is not None:
        cfg_path = os.path.join(path, "config.json")
        with open(cfg_path) as f:
            d = json.load(f)
        d["torch_dtype"] = d["dtype"] = name
        with open(cfg_path, "w") as f:
            json.dump(d, f, indent=2)
    # clone: q/k/v and gate/up share storage in this implementation
    sd = OrderedDict((k, v.detach().cpu().clone().contiguous()) for k, v in model.state_dict().items())
    if model.config.tie_word_embeddings:
        sd.pop("lm_head.weight", None)
    try:
        from safetensors.torch import save_file
    except ImportError:  # pragma: no cover
        torch.save(sd, os.path.join(path, "model.pt"))
        return
    save_file(sd, os.path.join(path, "model.safetensors"), metadata={"format": "pt"})


def _model_config(cfg) -> ModelConfig:
    mcfg = resolve_config(cfg.model.name)
    if mcfg.is_moe:
        mcfg.output_router_logits = bool(cfg.model.get("output_router_logits", True))
    return mcfg


def load_causal_lm(cfg, pconfig, dtype=torch.bfloat16, seed: int | None = None, device=None):
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
                                           seed=seed, device=device)
    return model, plan
