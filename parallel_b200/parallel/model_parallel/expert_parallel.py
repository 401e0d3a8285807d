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

import torch
import torch.distributed as dist

from ...ops.moe import LocalExpertTransport, routed_experts, routed_experts_supported
from ...profiling import collective_profile
from .token_dispatch import TokenDispatcher


class ExpertPartition:
    """Which experts an EP rank owns: the global expert ids are split into
    ``ep_size`` equal consecutive blocks and block ``r`` lives on rank ``r``
    (the layout the checkpoint plans and the route plan kernel assume).

    ``localize_routes`` maps global route ids to this rank's local ids; a
    route to another rank's expert becomes the sentinel ``local_count`` with
    score 0, which every expert kernel skips."""

    __slots__ = ("num_experts", "ep_size", "ep_rank", "local_count", "start", "stop")

    def __init__(self, num_experts: int, ep_size: int, ep_rank: int):
        per, rem = divmod(int(num_experts), max(int(ep_size), 1))
        problems = []
        if ep_size < 1:
            problems.append(f"the expert-parallel size is {ep_size}")
        elif rem:
            problems.append(f"{num_experts} experts do not split evenly over {ep_size} ranks")
        if ep_size >= 1 and not 0 <= ep_rank < ep_size:
            problems.append(f"rank {ep_rank} is not in an expert-parallel group of {ep_size}")
        if problems:
            raise ValueError("invalid expert partition: " + "; ".join(problems))
        self.num_experts, self.ep_size, self.ep_rank = int(num_experts), int(ep_size), int(ep_rank)
        self.local_count = per
        self.start, self.stop = ep_rank * per, (ep_rank + 1) * per

    def __repr__(self) -> str:
        return (f"ExpertPartition(experts [{self.start}, {self.stop}) of {self.num_experts} on rank "
                f"{self.ep_rank}/{self.ep_size})")

    def __eq__(self, other) -> bool:
        return isinstance(other, ExpertPartition) and (self.num_experts, self.ep_size, self.ep_rank) == (
            other.num_experts, other.ep_size, other.ep_rank)

    def __hash__(self) -> int:
        return hash((self.num_experts, self.ep_size, self.ep_rank))

    @property
    def global_experts(self) -> range:
        return range(self.start, self.stop)

    def owner(self, global_expert: torch.Tensor) -> torch.Tensor:
        """EP rank holding each global expert id."""
        return global_expert // self.local_count

    def localize_routes(self, global_indices: torch.Tensor, scores: torch.Tensor):
        """(local ids with the sentinel for foreign routes, scores with foreign
        routes zeroed, mask of the routes this rank computes)."""
        if global_indices.shape != scores.shape:
            raise ValueError(f"route ids {tuple(global_indices.shape)} and scores {tuple(scores.shape)} "
                             "differ in shape")
        mine = (global_indices >= self.start) & (global_indices < self.stop)
        local = torch.where(mine, global_indices - self.start, torch.full_like(global_indices, self.local_count))
        return local, torch.where(mine, scores, torch.zeros_like(scores)), mine


def local_expert_range(num_experts: int, ep_size: int, ep_rank: int) -> range:
    return ExpertPartition(num_experts, ep_size, ep_rank).global_experts


def verify_expert_modules(model, partition: ExpertPartition) -> None:
    """Every MoE block of the loaded model must hold exactly this rank's share
    of the experts (a model built for another EP size fails here)."""
    counts = {name: mod.num_experts for name, mod in model.named_modules()
              if name.endswith(".mlp.experts") and hasattr(mod, "num_experts")}
    if not counts:
        raise RuntimeError("expert parallelism is planned but the model has no '.mlp.experts' modules")
    wrong = {name: n for name, n in counts.items() if n != partition.local_count}
    if wrong:
        listed = ", ".join(f"{name} holds {n}" for name, n in sorted(wrong.items()))
        raise RuntimeError(f"each EP rank should hold {partition.local_count} experts per layer: {listed}")


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


class _ExpertRuntime:
    """Installs itself as the model's expert runtime (the MoE blocks call
    ``ctx.expert_runtime(experts, x, global_index, weights)``) and removes
    itself again; one model at a time."""

    _model = None

    def apply(self, model) -> None:
        if self._model is not None:
            raise RuntimeError(f"{type(self).__name__} is already installed on a model")
        model.ctx.expert_runtime = self
        model.set_parallel_context(model.ctx)
        self._model = model

    def close(self) -> None:
        model, self._model = self._model, None
        if model is not None:
            model.ctx.expert_runtime = None
            model.set_parallel_context(model.ctx)


class ReplicatedTokenExpertParallel(_ExpertRuntime):
    def __init__(self, partition: ExpertPartition, group, fused=None):
        self.partition = partition
        self.group = group
        # FusedTensorParallel of the TP group (NVLink all-reduces of the bf16
        # hidden states / expert outputs) or None
        self.fused = fused
        self.transport = LocalExpertTransport(partition.local_count, num_experts=partition.num_experts,
                                              ep_rank=partition.ep_rank, local_only=True)

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


class SequenceParallelExpertParallel(_ExpertRuntime):
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
