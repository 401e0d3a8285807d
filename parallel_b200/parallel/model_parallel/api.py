"""ModelParallelWrapper: activates TP / SP / EP on a local-shape model.

Same responsibilities and public methods as the reference wrapper
(parallel/parallel/engine/model_parallel/api.py:26-163): verify the model
against its plan, install the SUM_TP gradient reductions (one packed
all-reduce per decoder layer instead of one per parameter), switch on the sequence-
parallel runtime and the expert-parallel runtime, provide the vocab-parallel
token loss / training loss (+ router aux loss) and MP gradient clipping, and
own the checkpoint adapter (replaced by the composed one once FSDP is
attached).
"""
from __future__ import annotations

import torch

from ...models.qwen3 import ParallelContext
from . import comm_ops
from .fused_sp import FusedSequenceParallel, FusedTensorParallel
from .checkpoint import ComposedModelParallelCheckpoint, ModelParallelCheckpoint
from .expert_parallel import (ExpertPartition, ReplicatedTokenExpertParallel, SequenceParallelExpertParallel,
                              verify_expert_modules)
from .grad_norm import clip_grad_norm_
from .loss_parallel import loss_parallel_context, vocab_parallel_cross_entropy, vocab_parallel_lm_head_ce
from .registry import build_model_parallel_plan
from .sequence_parallel import SequenceParallelRuntime, sequence_parallel_load_balancing_loss
from .tensor_parallel import (install_layer_gradient_packs, install_tensor_parallel_gradient_hooks,
                              tensor_parallel_mesh, verify_tensor_parallel_model)


class ModelParallelWrapper:
    def __init__(self, model, pconfig, device, plan=None, collectives: str = "auto"):
        self.model = model
        self.pconfig = pconfig
        self.device = device
        self.plan = plan
        self.collectives = collectives
        self.mesh = None
        self.group = None
        self.experts = None
        self.expert_runtime = None
        self.sequence_runtime = None
        self.checkpoint = None
        self._tp_gradient_hook_handles = []
        self._replicated_ids: set[int] = set()
        if not self.is_active:
            return
        self.mesh = tensor_parallel_mesh(pconfig)
        self.group = self.mesh.get_group()
        if self.plan is None:
            self.plan = build_model_parallel_plan(model.config, pconfig)
        self.plan.validate_runtime(pconfig)
        if not hasattr(model, "_tp_size"):
            model._tp_size = getattr(model, "tp_size", 1)
        verify_tensor_parallel_model(model, self.plan, self.mesh)
        ctx = ParallelContext(tp_size=self.plan.tensor_parallel_size, tp_rank=self.mesh.get_local_rank(),
                              tp_group=self.group, sp=False, ep_size=self.plan.expert_parallel_size,
                              ep_rank=self.mesh.get_local_rank(), comm=comm_ops)
        model.set_parallel_context(ctx)
        # SUM_TP gradients: one packed reduction per decoder layer, per-param
        # hooks for the rest (the final norm under sequence parallelism)
        small = None
        if self.collectives != "nccl" and device is not None and torch.device(device).type == "cuda":
            from ..comm.p2p import P2PSmallAllReduce

            small = P2PSmallAllReduce.get(self.group, torch.device(device))
        packed = install_layer_gradient_packs(model, self.plan, self.mesh, small)
        self._tp_gradient_hook_handles = install_tensor_parallel_gradient_hooks(model, self.plan, self.mesh,
                                                                                exclude=packed)
        for name, p in model.named_parameters():
            if self.plan.placement_for_parameter(name).shard_dim is None:
                self._replicated_ids.add(id(p))
        if self.plan.capabilities.sequence_parallel:
            self.sequence_runtime = SequenceParallelRuntime(self.group,
                                                            dense_mlp=not self.plan.capabilities.expert_parallel)
            self.sequence_runtime.apply(model)
            # NVLink data plane: all-gather / reduce-scatter fused into the GEMMs
            if self.collectives != "nccl" and FusedSequenceParallel.available(self.group, device):
                ctx = model.ctx
                ctx.fused_tp = FusedSequenceParallel(self.group, device)
                model.set_parallel_context(ctx)
        elif self.collectives != "nccl" and FusedTensorParallel.available(self.group, device):
            # TP without SP: GEMM -> all-reduce over NVLink for the row-parallel outputs
            # and the column-parallel input gradients
            ctx = model.ctx
            ctx.fused_tp = FusedTensorParallel(self.group, device)
            model.set_parallel_context(ctx)
        if self.plan.capabilities.expert_parallel:
            self.experts = ExpertPartition(model.config.num_experts, self.plan.expert_parallel_size,
                                           self.mesh.get_local_rank())
            verify_expert_modules(model, self.experts)
            if self.plan.capabilities.sequence_parallel:
                self.expert_runtime = SequenceParallelExpertParallel(self.experts, self.group, device=device,
                                                                     collectives=self.collectives)
            else:
                fused = getattr(model.ctx, "fused_tp", None)
                self.expert_runtime = ReplicatedTokenExpertParallel(
                    self.experts, self.group, fused=fused if hasattr(fused, "try_all_reduce") else None)
            self.expert_runtime.apply(model)
        self.checkpoint = ModelParallelCheckpoint(model, pconfig, self.plan, self.mesh, device)

    @property
    def is_active(self) -> bool:
        return self.pconfig.model_parallel_enabled

    def backward_context(self):
        return loss_parallel_context(self.is_active)

    def token_loss(self, logits, labels, reduction: str = "mean"):
        if not self.is_active:
            return torch.nn.functional.cross_entropy(logits.reshape(-1, logits.shape[-1]).float(),
                                                     labels.reshape(-1), reduction=reduction)
        return vocab_parallel_cross_entropy(logits, labels, tp_mesh=self.mesh,
                                            vocab_size=self.model.config.vocab_size, reduction=reduction)

    def training_loss(self, outputs, labels):
        """Vocab-parallel CE on unshifted labels (+ router aux loss)."""
        h = getattr(outputs, "hidden_states", None)
        if outputs.logits is None and h is not None and h.is_cuda:
            loss = vocab_parallel_lm_head_ce(h, self.model.lm_head.weight, labels, self.group,
                                             self.model.vocab_start, collectives=self.collectives)
        else:
            logits = outputs.logits if outputs.logits is not None else self.model.lm_head(h)
            loss = self.token_loss(logits, labels)
        aux = getattr(outputs, "aux_loss", None)
        cfg = self.model.config
        if cfg.is_moe and cfg.output_router_logits:
            if self.plan.capabilities.sequence_parallel and self.plan.capabilities.expert_parallel:
                aux = sequence_parallel_load_balancing_loss(getattr(outputs, "router_logits", None),
                                                            num_experts=cfg.num_experts,
                                                            top_k=cfg.num_experts_per_tok, group=self.group,
                                                            collectives=self.collectives)
            else:
                from ...ops.moe import load_balancing_loss

                rl = getattr(outputs, "router_logits", None)
                aux = load_balancing_loss(rl, cfg.num_experts, cfg.num_experts_per_tok) if rl else None
            outputs.aux_loss = aux
        if aux is not None:
            loss = loss + cfg.router_aux_loss_coef * aux.to(loss.device)
        return loss

    def clip_grad_norm_(self, parameters, max_norm: float) -> torch.Tensor:
        if not self.is_active:
            return torch.nn.utils.clip_grad_norm_(parameters, max_norm)
        ids = {id(p) for p in parameters}
        named = [(n, p) for n, p in self._named_optimizer_params() if id(p) in ids]
        return clip_grad_norm_(named, max_norm, plan=self.plan, tp_mesh=self.mesh, pconfig=self.pconfig,
                               device=self.device)

    def _named_optimizer_params(self):
        return list(self.model.named_parameters())

    def is_replicated_param(self, p) -> bool:
        """True for parameters replicated over TP (counted once in the norm)."""
        if not self.is_active:
            return False
        if id(p) in self._replicated_ids:
            return True
        for n, q in self.model.named_parameters():
            if q is p:
                return self.plan.placement_for_parameter(n).shard_dim is None
        return False

    def replicated_grad_weight(self) -> float:
        return 1.0 if (not self.is_active or self.mesh.get_local_rank() == 0) else 0.0

    def full_state_dict(self):
        return self.checkpoint.full_state_dict()

    def load_full_state_dict(self, state_dict, strict: bool = True):
        return self.checkpoint.load_full_state_dict(state_dict, strict=strict)

    def sharded_state_dict(self):
        return self.checkpoint.sharded_state_dict()

    def load_sharded_state_dict(self, state_dict, strict: bool = True):
        return self.checkpoint.load_sharded_state_dict(state_dict, strict=strict)

    def checkpoint_layout(self):
        return self.checkpoint.checkpoint_layout()

    def attach_fsdp(self, fsdp_wrapper) -> None:
        if not self.is_active or not fsdp_wrapper.is_active:
            return
        # sharded DTensor params replace the full ones: remember which are replicated over TP
        for u in fsdp_wrapper.units:
            for m in u.param_metas:
                if id(m.parameter) in self._replicated_ids:
                    self._replicated_ids.add(id(m.sharded_param))
        self.checkpoint = ComposedModelParallelCheckpoint(self.model, self.pconfig, self.plan, self.mesh,
                                                          fsdp_wrapper, self.device)
