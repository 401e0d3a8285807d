"""Model configuration for the Qwen3 dense and Qwen3-MoE families.

Field names follow the Hugging Face ``config.json`` of these models, so a
config file written by ``save_pretrained`` (or one of the hub checkpoints)
loads directly, and configs written here load in HF.  The reference gets its
configs from ``AutoConfig.from_pretrained`` (parallel/parallel/engine/
model_loading.py:11-15).
"""
from __future__ import annotations

import dataclasses
import json
import os
from dataclasses import dataclass, field
from typing import Any


@dataclass
class ModelConfig:
    model_type: str = "qwen3"
    vocab_size: int = 151936
    hidden_size: int = 1024
    intermediate_size: int = 3072
    num_hidden_layers: int = 28
    num_attention_heads: int = 16
    num_key_value_heads: int = 8
    head_dim: int = 128
    rms_norm_eps: float = 1e-6
    rope_theta: float = 1_000_000.0
    max_position_embeddings: int = 40960
    tie_word_embeddings: bool = True
    attention_bias: bool = False
    hidden_act: str = "silu"
    initializer_range: float = 0.02
    torch_dtype: str = "bfloat16"
    # MoE (qwen3_moe)
    num_experts: int = 0
    num_experts_per_tok: int = 0
    moe_intermediate_size: int = 0
    norm_topk_prob: bool = False
    router_aux_loss_coef: float = 0.001
    output_router_logits: bool = False
    decoder_sparse_step: int = 1
    mlp_only_layers: list = field(default_factory=list)
    extra: dict = field(default_factory=dict)

    @property
    def is_moe(self) -> bool:
        return self.model_type == "qwen3_moe" and self.num_experts > 0

    def layer_is_moe(self, layer_idx: int) -> bool:
        return (
            self.is_moe
            and layer_idx not in self.mlp_only_layers
            and (layer_idx + 1) % self.decoder_sparse_step == 0
        )

    # ---- (de)serialisation -------------------------------------------------
    @classmethod
    def from_dict(cls, d: dict[str, Any]) -> "ModelConfig":
        names = {f.name for f in dataclasses.fields(cls)}
        kw = {k: v for k, v in d.items() if k in names and k != "extra"}
        extra = {k: v for k, v in d.items() if k not in names}
        rope = d.get("rope_parameters") or d.get("rope_scaling") or {}
        if "rope_theta" not in kw and isinstance(rope, dict) and "rope_theta" in rope:
            kw["rope_theta"] = rope["rope_theta"]
        if kw.get("head_dim") is None and "hidden_size" in kw:
            kw["head_dim"] = kw["hidden_size"] // kw.get("num_attention_heads", 16)
        cfg = cls(**kw)
        cfg.extra = extra
        return cfg

    @classmethod
    def from_pretrained(cls, path: str) -> "ModelConfig":
        with open(os.path.join(path, "config.json")) as f:
            return cls.from_dict(json.load(f))

    @classmethod
    def from_hf(cls, hf_config) -> "ModelConfig":
        return cls.from_dict(hf_config.to_dict())

    def to_dict(self) -> dict[str, Any]:
        d = dataclasses.asdict(self)
        extra = d.pop("extra", {}) or {}
        if not self.is_moe:
            for k in ("num_experts", "num_experts_per_tok", "moe_intermediate_size", "norm_topk_prob",
                      "router_aux_loss_coef", "output_router_logits", "decoder_sparse_step", "mlp_only_layers"):
                d.pop(k, None)
        d["architectures"] = ["Qwen3MoeForCausalLM" if self.is_moe else "Qwen3ForCausalLM"]
        d["rope_parameters"] = {"rope_type": "default", "rope_theta": self.rope_theta}
        d.update(extra)
        return d

    def save_pretrained(self, path: str) -> None:
        os.makedirs(path, exist_ok=True)
        with open(os.path.join(path, "config.json"), "w") as f:
            json.dump(self.to_dict(), f, indent=2)


# Named architectures used by the benchmarks (random-init weights).
PRESETS: dict[str, dict[str, Any]] = {
    "Qwen/Qwen3-0.6B": dict(model_type="qwen3", vocab_size=151936, hidden_size=1024, intermediate_size=3072,
                            num_hidden_layers=28, num_attention_heads=16, num_key_value_heads=8, head_dim=128,
                            tie_word_embeddings=True, max_position_embeddings=40960),
    "Qwen/Qwen3-8B": dict(model_type="qwen3", vocab_size=151936, hidden_size=4096, intermediate_size=12288,
                          num_hidden_layers=36, num_attention_heads=32, num_key_value_heads=8, head_dim=128,
                          tie_word_embeddings=False, max_position_embeddings=40960),
    "Qwen/Qwen3-30B-A3B": dict(model_type="qwen3_moe", vocab_size=151936, hidden_size=2048,
                               intermediate_size=6144, num_hidden_layers=48, num_attention_heads=32,
                               num_key_value_heads=4, head_dim=128, num_experts=128, num_experts_per_tok=8,
                               moe_intermediate_size=768, norm_topk_prob=True, router_aux_loss_coef=0.001,
                               tie_word_embeddings=False, max_position_embeddings=40960),
    # small configs with head_dim 128 (the attention kernels' head size) for GPU tests
    "small-qwen3": dict(model_type="qwen3", vocab_size=2048, hidden_size=256, intermediate_size=512,
                        num_hidden_layers=2, num_attention_heads=4, num_key_value_heads=2, head_dim=128,
                        tie_word_embeddings=True),
    "small-qwen3-moe": dict(model_type="qwen3_moe", vocab_size=2048, hidden_size=256, intermediate_size=512,
                            num_hidden_layers=2, num_attention_heads=4, num_key_value_heads=2, head_dim=128,
                            num_experts=8, num_experts_per_tok=2, moe_intermediate_size=128, norm_topk_prob=True,
                            tie_word_embeddings=False, output_router_logits=True),
    # tiny configs for tests
    "tiny-qwen3": dict(model_type="qwen3", vocab_size=1024, hidden_size=256, intermediate_size=512,
                       num_hidden_layers=2, num_attention_heads=4, num_key_value_heads=2, head_dim=64,
                       tie_word_embeddings=True),
    "tiny-qwen3-moe": dict(model_type="qwen3_moe", vocab_size=1024, hidden_size=256, intermediate_size=512,
                           num_hidden_layers=2, num_attention_heads=4, num_key_value_heads=2, head_dim=64,
                           num_experts=4, num_experts_per_tok=2, moe_intermediate_size=128,
                           tie_word_embeddings=False, output_router_logits=True),
}


def resolve_config(name_or_path: str, **overrides) -> ModelConfig:
    """A local HF directory, a preset name, or a hub id that matches a preset."""
    if os.path.isdir(name_or_path) and os.path.exists(os.path.join(name_or_path, "config.json")):
        cfg = ModelConfig.from_pretrained(name_or_path)
    elif name_or_path in PRESETS:
        cfg = ModelConfig.from_dict(dict(PRESETS[name_or_path]))
    else:
        raise FileNotFoundError(
            f"Unknown model {name_or_path!r}: pass a local directory with config.json or one of {sorted(PRESETS)}"
        )
    for k, v in overrides.items():
        setattr(cfg, k, v)
    return cfg
