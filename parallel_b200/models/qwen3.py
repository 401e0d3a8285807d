"""Qwen3 dense and Qwen3-MoE causal LMs built on the fused sm_100a ops.

The module tree and parameter names are the Hugging Face ones
(``model.embed_tokens.weight``, ``model.layers.{i}.self_attn.q_proj.weight``,
``...mlp.gate.weight``, ``...mlp.experts.gate_up_proj`` [E, 2I, H] with the
gate half first, ``...mlp.experts.down_proj`` [E, H, I], ``lm_head.weight``)
so portable checkpoints interchange with HF and with the reference, which
trains the HF modules directly (parallel/parallel/engine/model_loading.py).

Tensor / sequence / expert parallelism is carried by a ``ParallelContext``
set by the model-parallel wrapper: with it the modules hold local shards
(heads, MLP columns, vocab rows, experts) and insert the collectives of the
reference's HF TP styles (parallel/parallel/engine/model_parallel/
tensor_parallel.py, sequence_parallel.py, expert_parallel.py).
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import Any, Optional

import torch
import torch.nn as nn

from ..ops import functional as Fx
from ..ops import moe as MoE
from .config import ModelConfig


@dataclass
class ParallelContext:
    """Model-parallel facts the modules need; all defaults = single device."""

    tp_size: int = 1
    tp_rank: int = 0
    tp_group: Any = None
    sp: bool = False
    ep_size: int = 1
    ep_rank: int = 0
    expert_runtime: Any = None  # ReplicatedTokenExpertParallel / SequenceParallelExpertParallel
    comm: Any = None  # model_parallel.comm_ops module (set by the wrapper)
    # NVLink GEMM + collective data plane of the TP group: FusedSequenceParallel
    # under sequence parallelism, FusedTensorParallel without it, or None
    fused_tp: Any = None

    @property
    def active(self) -> bool:
        return self.tp_size > 1


@dataclass
class CausalLMOutput:
    loss: Optional[torch.Tensor] = None
    logits: Optional[torch.Tensor] = None
    aux_loss: Optional[torch.Tensor] = None
    router_logits: Optional[tuple] = None
    hidden_states: Optional[torch.Tensor] = None


class RMSNorm(nn.Module):
    def __init__(self, dim: int, eps: float = 1e-6):
        super().__init__()
        self.weight = nn.Parameter(torch.ones(dim))
        self.variance_epsilon = eps

    def forward(self, x):
        return Fx.rms_norm(x, self.weight, self.variance_epsilon)


class Linear(nn.Module):
    """Bias-free linear layer holding ``weight`` [out, in] (HF name)."""

    def __init__(self, in_features: int, out_features: int):
        super().__init__()
        self.in_features, self.out_features = in_features, out_features
        self.weight = nn.Parameter(torch.empty(out_features, in_features))

    def forward(self, x, residual=None):
        return Fx.linear(x, self.weight, residual)


class Embedding(nn.Module):
    def __init__(self, num: int, dim: int):
        super().__init__()
        self.weight = nn.Parameter(torch.empty(num, dim))

    def forward(self, ids, vocab_start: int = 0, tied=None):
        # an FSDP wrapper may install a one-shot reader that fetches the rows of
        # this batch from the row shards while the full table is still being gathered
        reader = self.__dict__.pop("_sharded_lookup", None)
        return Fx.embedding(ids, self.weight, vocab_start, tied, reader=reader)


class RotaryEmbedding(nn.Module):
    def __init__(self, cfg: ModelConfig):
        super().__init__()
        D = cfg.head_dim
        inv = 1.0 / (cfg.rope_theta ** (torch.arange(0, D, 2, dtype=torch.int64).float() / D))
        self.register_buffer("inv_freq", inv, persistent=False)


class Attention(nn.Module):
    def __init__(self, cfg: ModelConfig, layer_idx: int, tp: int = 1):
        super().__init__()
        D = cfg.head_dim
        self.layer_idx = layer_idx
        self.head_dim = D
        self.num_heads = cfg.num_attention_heads // tp
        self.num_kv_heads = cfg.num_key_value_heads // tp
        self.eps = cfg.rms_norm_eps
        H = cfg.hidden_size
        self.q_proj = Linear(H, self.num_heads * D)
        self.k_proj = Linear(H, self.num_kv_heads * D)
        self.v_proj = Linear(H, self.num_kv_heads * D)
        self.o_proj = Linear(self.num_heads * D, H)
        self.q_norm = RMSNorm(D, cfg.rms_norm_eps)
        self.k_norm = RMSNorm(D, cfg.rms_norm_eps)

    def core(self, h, inv_freq, B, S, stash=None, sp=None):
        """Attention output before o_proj: [B*S, heads*D].  With ``sp`` (fused
        sequence parallel), h is this rank's sequence shard and the all-gather
        runs inside the QKV GEMM."""
        return Fx.attention_block(h, self.q_proj.weight, self.k_proj.weight, self.v_proj.weight,
                                  self.q_norm.weight, self.k_norm.weight, inv_freq, B, S, self.num_heads,
                                  self.num_kv_heads, self.head_dim, self.eps, stash, sp)


class MLP(nn.Module):
    def __init__(self, cfg: ModelConfig, intermediate: int, tp: int = 1):
        super().__init__()
        H = cfg.hidden_size
        I = intermediate // tp
        self.gate_proj = Linear(H, I)
        self.up_proj = Linear(H, I)
        self.down_proj = Linear(I, H)

    def forward(self, x, residual=None, output_unused: bool = False):
        return Fx.swiglu_mlp(x, self.gate_proj.weight, self.up_proj.weight, self.down_proj.weight, residual,
                             output_unused)


class TopKRouter(nn.Module):
    """HF Qwen3MoeTopKRouter: fp32 softmax over x W^T, top-k, optional renorm."""

    def __init__(self, cfg: ModelConfig):
        super().__init__()
        self.top_k = cfg.num_experts_per_tok
        self.num_experts = cfg.num_experts
        self.norm_topk_prob = cfg.norm_topk_prob
        self.weight = nn.Parameter(torch.zeros(cfg.num_experts, cfg.hidden_size))
        # optional per-expert logit offset (not part of the model's state: a
        # benchmark knob that skews routing, e.g. N(0, 2) for the skewed-router
        # workload); None means the plain HF router
        self.logit_bias: torch.Tensor | None = None

    def forward(self, x):
        return MoE.route(x.reshape(-1, x.shape[-1]), self.weight, self.top_k, self.norm_topk_prob,
                         logit_bias=self.logit_bias)


class Experts(nn.Module):
    def __init__(self, cfg: ModelConfig, num_local: int):
        super().__init__()
        self.num_experts = num_local
        self.intermediate_dim = cfg.moe_intermediate_size
        self.gate_up_proj = nn.Parameter(torch.empty(num_local, 2 * cfg.moe_intermediate_size, cfg.hidden_size))
        self.down_proj = nn.Parameter(torch.empty(num_local, cfg.hidden_size, cfg.moe_intermediate_size))

    def forward(self, x, top_k_index, top_k_weights):
        return MoE.experts_forward(x, top_k_index, top_k_weights, self.gate_up_proj, self.down_proj)


class SparseMoeBlock(nn.Module):
    def __init__(self, cfg: ModelConfig, ep: int = 1):
        super().__init__()
        # registration order = HF's (experts, then the router): the FSDP bucket
        # layout follows parameter order, so exact-topology checkpoints depend on it
        self.experts = Experts(cfg, cfg.num_experts // ep)
        self.gate = TopKRouter(cfg)
        self.num_experts = cfg.num_experts
        self.top_k = cfg.num_experts_per_tok

    def forward(self, x, ctx: ParallelContext, router_sink: list):
        shape = x.shape
        x2 = x.reshape(-1, shape[-1])
        probs, weights, index = self.gate(x2)
        router_sink.append(probs)
        if ctx.expert_runtime is not None:
            y = ctx.expert_runtime(self.experts, x2, index, weights)
        else:
            y = self.experts(x2, index, weights)
        return y.reshape(shape)


class DecoderLayer(nn.Module):
    def __init__(self, cfg: ModelConfig, layer_idx: int, tp: int = 1, ep: int = 1):
        super().__init__()
        self.layer_idx = layer_idx
        self.self_attn = Attention(cfg, layer_idx, tp)
        self.is_moe = cfg.layer_is_moe(layer_idx)
        if self.is_moe:
            self.mlp = SparseMoeBlock(cfg, ep)
        else:
            self.mlp = MLP(cfg, cfg.intermediate_size, tp)
        self.input_layernorm = RMSNorm(cfg.hidden_size, cfg.rms_norm_eps)
        self.post_attention_layernorm = RMSNorm(cfg.hidden_size, cfg.rms_norm_eps)
        self._ctx = ParallelContext()
        self._router_sink: list = []
        self._inv_freq = None
        self._seq = None
        # model parallelism: the layer's TP-summed parameters, their gradients
        # reduced in one collective (set by the model-parallel wrapper)
        self._tp_grad_pack = None

    def forward(self, x):
        """x: [B, S_local, H] (S_local = S / tp under sequence parallelism)."""
        pack = self._tp_grad_pack
        if pack is not None and torch.is_grad_enabled():
            return pack.run(self._forward, x)
        return self._forward(x)

    def _forward(self, x):
        ctx = self._ctx
        B, S = self._seq
        stash = getattr(self, "_attn_stash", None)
        fsp = ctx.fused_tp if (ctx.tp_size > 1 and ctx.fused_tp is not None and x.is_cuda
                               and ctx.fused_tp.supports(B, S, x.shape[-1])) else None
        if fsp is not None:
            # tensor / sequence parallel on the fused NVLink kernels: the gathers run
            # inside the column-parallel GEMMs, the reduce-scatters (all-reduces
            # without SP) inside the row-parallel ones
            from ..parallel.model_parallel.fused_sp import linear_reduce_scatter, sp_swiglu_mlp

            h = self.input_layernorm(x)
            o = self.self_attn.core(h, self._inv_freq, B, S, stash, sp=fsp)
            y = linear_reduce_scatter(o, self.self_attn.o_proj.weight, fsp, B, S)
            x = x + y.view(x.shape)
            h = self.post_attention_layernorm(x)
            if self.is_moe:
                return x + self.mlp(h, ctx, self._router_sink)
            return x + sp_swiglu_mlp(h, self.mlp.gate_proj.weight, self.mlp.up_proj.weight,
                                     self.mlp.down_proj.weight, fsp, B, S)
        if ctx.tp_size > 1:
            h = self.input_layernorm(x)
            h = ctx.comm.gather_sequence(h, ctx) if ctx.sp else ctx.comm.copy_to_tp(h, ctx)
            o = self.self_attn.core(h, self._inv_freq, B, S, stash)
            y = self.self_attn.o_proj(o).view(B, S, -1)
            y = ctx.comm.reduce_scatter_sequence(y, ctx) if ctx.sp else ctx.comm.reduce_from_tp(y, ctx)
            x = x + y
            h = self.post_attention_layernorm(x)
        else:
            x_res, h = Fx.residual_rms_norm(x, self.input_layernorm.weight, self.input_layernorm.variance_epsilon)
            o = self.self_attn.core(h, self._inv_freq, B, S, stash)
            x = self.self_attn.o_proj(o, residual=x_res)
            x, h = Fx.residual_rms_norm(x, self.post_attention_layernorm.weight,
                                        self.post_attention_layernorm.variance_epsilon)
        if self.is_moe:
            return x + self.mlp(h, ctx, self._router_sink)
        if ctx.tp_size > 1:
            h = ctx.comm.gather_sequence(h, ctx) if ctx.sp else ctx.comm.copy_to_tp(h, ctx)
            y = self.mlp(h)
            y = ctx.comm.reduce_scatter_sequence(y, ctx) if ctx.sp else ctx.comm.reduce_from_tp(y, ctx)
            return x + y
        # in an activation-checkpoint recompute the layer output only carries
        # the gradient (the FSDP unit differentiates through it), so the final
        # down projection is skipped there
        return self.mlp(h, residual=x, output_unused=getattr(self, "_recomputing", False))


class Qwen3Model(nn.Module):
    def __init__(self, cfg: ModelConfig, tp: int = 1, ep: int = 1):
        super().__init__()
        self.config = cfg
        self.vocab_size = cfg.vocab_size
        self.embed_tokens = Embedding(cfg.vocab_size // tp, cfg.hidden_size)
        self.layers = nn.ModuleList(DecoderLayer(cfg, i, tp, ep) for i in range(cfg.num_hidden_layers))
        self.norm = RMSNorm(cfg.hidden_size, cfg.rms_norm_eps)
        self.rotary_emb = RotaryEmbedding(cfg)


class Qwen3ForCausalLM(nn.Module):
    """Qwen3 / Qwen3-MoE causal LM (``config.model_type`` selects the MLP)."""

    def __init__(self, config: ModelConfig, tp: int = 1, ep: int = 1, device=None, dtype=None):
        super().__init__()
        self.config = config
        self.tp_size, self.ep_size = tp, ep
        self.model = Qwen3Model(config, tp, ep)
        self.lm_head = Linear(config.hidden_size, config.vocab_size // tp)
        if config.tie_word_embeddings:
            self.lm_head.weight = self.model.embed_tokens.weight
        self.ctx = ParallelContext()
        if dtype is not None or device is not None:
            self.to(device=device, dtype=dtype)
        self._layout_fused_weights()

    # HF-compatible attribute used by checkpoint code
    _tied_weights_keys = {"lm_head.weight": "model.embed_tokens.weight"}

    def _layout_fused_weights(self):
        """Give q/k/v and gate/up adjacent storage so the fused GEMMs read
        them as one matrix without copies."""
        for layer in self.model.layers:
            a = layer.self_attn
            _share_storage([a.q_proj, a.k_proj, a.v_proj])
            if isinstance(layer.mlp, MLP):
                _share_storage([layer.mlp.gate_proj, layer.mlp.up_proj])

    def set_parallel_context(self, ctx: ParallelContext):
        self.ctx = ctx
        for layer in self.model.layers:
            layer._ctx = ctx

    @property
    def vocab_start(self) -> int:
        return self.ctx.tp_rank * (self.config.vocab_size // self.ctx.tp_size) if self.ctx.tp_size > 1 else 0

    def init_weights(self, seed: int | None = None, std: float | None = None):
        """HF ``_init_weights``: normal(0, initializer_range) for matrices,
        ones for norms."""
        std = self.config.initializer_range if std is None else std
        gen = None
        dev = next(self.parameters()).device
        if seed is not None:
            # the draw follows the parameters' device: a model built on the GPU
            # (large benchmark models) draws there, one parameter at a time
            gen = torch.Generator(device=dev).manual_seed(seed)
        with torch.no_grad():
            for name, p in self.named_parameters():
                if name.endswith("norm.weight") or ".q_norm." in name or ".k_norm." in name or "layernorm" in name:
                    p.fill_(1.0)
                else:
                    if gen is not None:
                        p.copy_(torch.randn(p.shape, generator=gen, dtype=torch.float32, device=dev) * std)
                    else:
                        p.normal_(0.0, std)

    def forward(self, input_ids: torch.Tensor, labels: torch.Tensor | None = None, shift_labels: bool = True,
                return_logits: bool = False, output_router_logits: bool | None = None) -> CausalLMOutput:
        ctx = self.ctx
        B, S = input_ids.shape
        inv_freq = self.model.rotary_emb.inv_freq
        for layer in self.model.layers:
            layer._seq = (B, S)
            layer._inv_freq = inv_freq
            layer._router_sink = []
        # tied embedding / LM head on the fused CE path: the embedding backward
        # updates the LM head's weight gradient in place
        tied = (Fx.TiedGrad() if self.config.tie_word_embeddings and ctx.tp_size == 1 and labels is not None
                and input_ids.is_cuda else None)
        x = self.model.embed_tokens(input_ids, self.vocab_start, tied)
        if ctx.tp_size > 1:
            x = ctx.comm.reduce_from_tp(x, ctx)
            if ctx.sp:
                x = ctx.comm.scatter_sequence(x, ctx)
        for layer in self.model.layers:
            x = layer(x)
        x = self.model.norm(x)
        router_logits = tuple(p for layer in self.model.layers for p in layer._router_sink)
        for layer in self.model.layers:
            layer._router_sink = []
        out = CausalLMOutput(router_logits=router_logits if router_logits else None)
        if ctx.tp_size > 1:
            # model-parallel path: logits stay vocab-sharded; the wrapper's
            # training_loss computes the vocab-parallel CE (no label shift)
            if ctx.sp:
                x = ctx.comm.gather_sequence(x, ctx)
            else:
                x = ctx.comm.copy_to_tp(x, ctx)
            out.hidden_states = x
            if return_logits or (labels is None and not x.is_cuda):
                out.logits = self.lm_head(x)
            return out
        if labels is not None:
            y = Fx.shift_labels(labels) if shift_labels else labels
            out.loss = Fx.lm_head_cross_entropy(x.reshape(B * S, -1), self.lm_head.weight, y, tied=tied)
            if self.config.is_moe and (self.config.output_router_logits if output_router_logits is None
                                       else output_router_logits) and router_logits:
                out.aux_loss = MoE.load_balancing_loss(router_logits, self.config.num_experts,
                                                       self.config.num_experts_per_tok)
                out.loss = out.loss + self.config.router_aux_loss_coef * out.aux_loss
        if return_logits or labels is None:
            out.logits = self.lm_head(x)
        out.hidden_states = x
        return out


def _share_storage(linears: list) -> None:
    """Re-home the weights of ``linears`` into one contiguous buffer
    (row-concatenated, registration order)."""
    ws = [l.weight for l in linears]
    if any(w.is_meta for w in ws):
        return
    dtype, device = ws[0].dtype, ws[0].device
    if any(w.dtype != dtype or w.device != device or w.shape[1] != ws[0].shape[1] for w in ws):
        return
    buf = torch.cat([w.detach() for w in ws], 0)
    r = 0
    for l, w in zip(linears, ws):
        n = w.shape[0]
        l.weight = nn.Parameter(buf[r:r + n], requires_grad=w.requires_grad)
        r += n


def build_model(config: ModelConfig, device=None, dtype=torch.bfloat16, tp: int = 1, ep: int = 1,
                seed: int | None = None) -> Qwen3ForCausalLM:
    """Random-init (HF init) model on ``device`` in ``dtype``."""
    model = Qwen3ForCausalLM(config, tp=tp, ep=ep)
    model.init_weights(seed=seed)
    model.to(dtype=dtype)
    if device is not None:
        model.to(device)
    model._layout_fused_weights()
    return model
