"""Expert parallelism folded onto the TP ranks.

* ``ExpertPartition``: contiguous ownership ``owner = e // local_count`` and
  route localisation (non-local routes get the sentinel index
  ``local_count`` and score 0).
* ``ReplicatedTokenExpertParallel`` (no SP): every rank routes all tokens,
  runs its local experts, and the expert output is all-reduced (forward);
  hidden-state and score gradients are all-reduced in backward.
* ``SequenceParallelExpertParallel`` (SP): each rank's local tokens are
  dispatched to the expert owners with variable all-to-alls and combined
  back.

Semantics: parallel/parallel/engine/model_parallel/expert_parallel.py.  The
runtimes are callables the MoE block invokes as
``runtime(experts, x, global_index, weights)``.
"""
from __future__ import annotations

from dataclasses import dataclass

import torch
import torch.distributed as dist

from ...ops.moe import LocalExpertTransport, routed_experts, routed_experts_supported
from ...profiling import collective_profile
from .token_dispatch import TokenDispatcher


@dataclass(frozen=True)
class ExpertPartition:
    num_experts: int
    ep_size: int
    ep_rank: int

    def __post_init__(self):
        if self.ep_size < 1:
            raise ValueError("ep_size must be positive")
        if not 0 <= self.ep_rank < self.ep_size:
            raise ValueError("ep_rank is outside the expert-parallel group")
        if self.num_experts % self.ep_size:
            raise ValueError(f"num_experts ({self.num_experts}) must be divisible by ep_size ({self.ep_size})")

    @property
    def local_count(self) -> int:
        return self.num_experts // self.ep_size

    @property
    def start(self) -> int:
        return self.ep_rank * self.local_count

    @property
    def stop(self) -> int:
        return self.start + self.local_count

    @property
    def global_experts(self) -> range:
        return range(self.start, self.stop)

    def owner(self, global_expert: torch.Tensor) -> torch.Tensor:
        return torch.div(global_expert, self.local_count, rounding_mode="floor")

    def localize_routes(self, global_indices: torch.Tensor, scores: torch.Tensor):
        if global_indices.shape != scores.shape:
            raise ValueError("Expert indices and scores must have the same shape")
        local_mask = self.owner(global_indices) == self.ep_rank
        local_idx = (global_indices - self.start).masked_fill(~local_mask, self.local_count)
        return local_idx, scores.masked_fill(~local_mask, 0), local_mask


def local_expert_range(num_experts: int, ep_size: int, ep_rank: int) -> range:
    return ExpertPartition(num_experts, ep_size, ep_rank).global_experts


def verify_expert_modules(model, partition: ExpertPartition) -> None:
    mods = [(n, m) for n, m in model.named_modules() if n.endswith(".mlp.experts") and hasattr(m, "num_experts")]
    if not mods:
        raise RuntimeError("Expert-parallel plan found no expert modules")
    bad = [f"{n}={m.num_experts}" for n, m in mods if m.num_experts != partition.local_count]
    if bad:
        raise RuntimeError(f"Expected {partition.local_count} local experts per rank, got " + ", ".join(bad))


def _sum(value, group, fused, mode):
    """SUM over the group: NVLink peer memory through ``fused`` (a
    FusedTensorParallel) when the tensor fits it, NCCL / gloo otherwise."""
    if fused is not None:
        out = fused.try_all_reduce(value)
        if out is not None:
            return out
    out = value.contiguous().clone()
    with collective_profile("ep_all_reduce", value=out, mode=mode, detail="expert_boundary"):
        dist.all_reduce(out, op=dist.ReduceOp.SUM, group=group)
    return out


class _AllReduceBackward(torch.autograd.Function):
    @staticmethod
    def forward(ctx, value, group, fused=None):
        ctx.group, ctx.fused = group, fused
        return value

    @staticmethod
    def backward(ctx, g):
        return _sum(g, ctx.group, ctx.fused, "replicated_token_grad"), None, None


class _AllReduceForward(torch.autograd.Function):
    @staticmethod
    def forward(ctx, value, group, fused=None):
        return _sum(value, group, fused, "replicated_token_output")

    @staticmethod
    def backward(ctx, g):
        return g, None, None


class ReplicatedTokenExpertParallel:
    def __init__(self, partition: ExpertPartition, group, fused=None):
        self.partition = partition
        self.group = group
        # FusedTensorParallel of the TP group (NVLink all-reduces of the bf16
        # hidden states / expert outputs) or None
        self.fused = fused
        self.transport = LocalExpertTransport(partition.local_count, num_experts=partition.num_experts,
                                              ep_rank=partition.ep_rank, local_only=True)
        self._model = None

    def __call__(self, experts, x2, global_index, weights):
        # the routing weights pass the backward all-reduce boundary before they
        # are localised, so every rank's weight gradient sums into each route
        weights = _AllReduceBackward.apply(weights, self.group)
        h = _AllReduceBackward.apply(x2, self.group, self.fused)
        if routed_experts_supported(h, experts.gate_up_proj, self.partition.num_experts):
            # device path: routes to other ranks' experts are dropped by the plan
            y = routed_experts(h, weights, global_index, experts.gate_up_proj, experts.down_proj, self.transport)
        else:
            local_idx, local_w, _ = self.partition.localize_routes(global_index, weights)
            y = experts(h, local_idx, local_w)
        return _AllReduceForward.apply(y, self.group, self.fused)

    def apply(self, model) -> None:
        if self._model is not None:
            raise RuntimeError("Expert parallel hooks are already installed")
        ctx = model.ctx
        ctx.expert_runtime = self
        model.set_parallel_context(ctx)
        self._model = model

    def close(self) -> None:
        if self._model is not None:
            self._model.ctx.expert_runtime = None
            self._model.set_parallel_context(self._model.ctx)
            self._model = None


class SequenceParallelExpertParallel:
    def __init__(self, partition: ExpertPartition, group, device=None, collectives: str = "auto"):
        self.partition = partition
        self.group = group
        # NVLink peer memory with a device-resident routing plan on CUDA (<= 8
        # ranks); variable all-to-alls with host-read split sizes otherwise
        from .p2p_dispatch import PeerExpertTransport

        self.transport = None
        if device is not None and collectives != "nccl" and PeerExpertTransport.available(group, device):
            self.transport = PeerExpertTransport(partition, group, device)
        self.dispatcher = TokenDispatcher(partition, group)
        self._model = None

    def __call__(self, experts, x2, global_index, weights):
        if self.transport is not None and routed_experts_supported(x2, experts.gate_up_proj,
                                                                   self.partition.num_experts):
            return routed_experts(x2, weights, global_index, experts.gate_up_proj, experts.down_proj, self.transport)
        hidden, idx, w, state = self.dispatcher.dispatch(x2, global_index, weights)
        y = experts(hidden, idx, w)
        return self.dispatcher.combine(y, state)

    def apply(self, model) -> None:
        if self._model is not None:
            raise RuntimeError("Expert parallel hooks are already installed")
        ctx = model.ctx
        ctx.expert_runtime = self
        model.set_parallel_context(ctx)
        self._model = model

    def close(self) -> None:
        if self._model is not None:
            self._model.ctx.expert_runtime = None
            self._model.set_parallel_context(self._model.ctx)
            self._model = None
