"""Fully sharded data parallelism over flat per-layer units.

Public surface mirrors the reference FSDPWrapper (parallel/parallel/engine/
dp_sharded.py:22-886): ``shard_model``, ``prepare_backward``,
``finalize_backward``, ``get_optimizer_params``, ``clip_grad_norm_``, the
full / local-full / sharded state-dict methods and ``checkpoint_layout``
(same dict, so exact-topology checkpoints interchange).

Execution model (B200-first):
* each decoder layer runs through one autograd Function (``_UnitFn``) that
  gathers the unit (or waits for the side-stream prefetch), starts the next
  prefetch, runs the layer - under ``no_grad`` when activation checkpointing
  is on, recomputing it in backward - and, in backward, produces the unit's
  full gradients with one ``torch.autograd.grad`` call and immediately
  launches its reduce-scatter.  Reductions therefore leave in strict reverse
  unit order on every rank with at most two in flight, exactly the
  reference's schedule, without per-parameter hooks;
* the root unit (embedding, final norm, untied LM head) is gathered at the
  start of forward and kept until the end of backward
  (reshard_after_forward=False), as in the reference;
* with ``find_unused_parameters`` the reductions are issued after backward
  in fixed order (zeros for units/parameters without a local gradient) and
  a participation bitmap all-reduced over the shard group decides which
  parameters receive a gradient (globally unused ones keep ``grad=None``,
  so AdamW skips them, as in the reference).
"""
from __future__ import annotations

import os
from typing import Any, Optional

import torch
import torch.distributed as dist
import torch.nn as nn

from ..state import Strategies
from .comm.unit_collectives import make_unit_collectives
from .fsdp_state import FSDPStateMixin
from .fsdp_utils import get_fsdp_units, group_named_parameters, local_tensor
from .param_unit import DPParamUnit


def _sink_of(unit):
    return getattr(unit.module, "_router_sink", None)


def _run_layer(unit, fwd, x, args):
    """Run the layer; returns (y, extras) where extras are the tensors the
    layer appended to its router sink (MoE router probabilities, which feed
    the auxiliary loss and so must stay differentiable)."""
    sink = _sink_of(unit)
    n0 = len(sink) if sink is not None else 0
    y = fwd(x, *args)
    extras = []
    if sink is not None and len(sink) > n0:
        extras = list(sink[n0:])
        del sink[n0:]
    return y, extras


class _UnitFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, wrapper, unit, fwd, nargs, x, *args):
        unit.all_gather()
        if unit.next_fwd is not None:
            unit.next_fwd.prefetch()
        if unit.use_activation_checkpoint:
            # selective recompute: the layer keeps its attention output from
            # this pass and reuses it when it is recomputed in backward
            unit.module._attn_stash = {"mode": "save"} if wrapper.keep_attention_output else None
            with torch.no_grad():
                y, extras = _run_layer(unit, fwd, x, args)
            ctx.stash = unit.module._attn_stash
            unit.module._attn_stash = None
            ctx.save_for_backward(x)
            ctx.inner = None
        else:
            xi = x.detach().requires_grad_(True)
            with torch.enable_grad():
                y, extras = _run_layer(unit, fwd, xi, args)
            ctx.inner = (xi, y, extras)
            y = y.detach()
            extras = [e.detach() for e in extras]
        if unit.reshard_after_forward:
            unit.free_full_params()
        ctx.wrapper, ctx.unit, ctx.fwd, ctx.args = wrapper, unit, fwd, args
        ctx.n_extra = len(extras)
        return (y, *extras)

    @staticmethod
    def backward(ctx, gy, *gextras):
        wrapper, unit = ctx.wrapper, ctx.unit
        unit.all_gather()
        if unit.next_bwd is not None:
            unit.next_bwd.prefetch()
        if ctx.inner is None:
            (x,) = ctx.saved_tensors
            xi = x.detach().requires_grad_(True)
            stash = getattr(ctx, "stash", None)
            if stash is not None:
                stash["mode"] = "reuse"
            unit.module._attn_stash = stash
            # the recomputed output only carries gy into autograd.grad below:
            # layers may skip computing its value (the dense MLP's down GEMM)
            unit.module._recomputing = True
            try:
                with torch.enable_grad():
                    y, extras = _run_layer(unit, ctx.fwd, xi, ctx.args)
            finally:
                unit.module._attn_stash = None
                unit.module._recomputing = False
                ctx.stash = None
        else:
            xi, y, extras = ctx.inner
        ctx.inner = None
        outs, gouts = [y], [gy]
        for e, g in zip(extras, gextras):
            if g is not None and e.requires_grad:
                outs.append(e)
                gouts.append(g)
        params = unit.parameters if unit.requires_grad else []
        grads = torch.autograd.grad(outs, [xi] + params, gouts, allow_unused=True)
        del y, extras, outs
        if unit.requires_grad:
            wrapper._unit_backward_done(unit, list(grads[1:]))
        else:
            unit.free_full_params()
        return (None, None, None, None, grads[0]) + (None,) * len(ctx.args)


class FSDPWrapper(FSDPStateMixin):
    """FSDP over ``model.model.layers`` plus a root unit (see module docstring)."""

    def __init__(self, model: nn.Module, pconfig, cpu_offload: bool = False, activation_checkpoint: bool = False,
                 checkpoint_every_n: int = 1, find_unused_parameters: bool = False,
                 overlap_backward_reductions: bool = True, device: Optional[torch.device] = None,
                 collectives: str = "auto"):
        self.model = model
        self.pconfig = pconfig
        self.cpu_offload = cpu_offload
        self.activation_checkpoint = activation_checkpoint
        self.checkpoint_every_n = max(checkpoint_every_n, 1)
        self.find_unused_parameters = find_unused_parameters
        self.overlap_backward_reductions = overlap_backward_reductions
        first = next(model.parameters(), None)
        self.device = device or (first.device if first is not None else torch.device("cpu"))
        self.collectives_kind = collectives
        # under activation checkpointing keep each layer's attention output
        # (and log-sum-exp) so the backward recompute skips the attention kernel
        self.keep_attention_output = True
        self.units: list[DPParamUnit] = []
        self.root_units: list[DPParamUnit] = []
        self.dp_shard_group = None
        self.dp_shard_mesh = None
        self._inflight: list[DPParamUnit] = []
        self._max_inflight = 2
        self._backward_prepared = False
        self._done_units: set[int] = set()
        self._deferred: dict[int, list] = {}
        self.state_keys: tuple[str, ...] = ()
        self.state_names: dict[int, tuple[str, ...]] = {}
        self.param_keys: set[str] = set()
        self._orig_forwards: dict[int, Any] = {}
        self._root_hook = None
        self.coll = None

    # ------------------------------------------------------------------ sharding
    def shard_model(self):
        self._index_state()
        if self.pconfig.dp_shard_size <= 1 or self.pconfig.device_mesh is None:
            return
        if self.units:
            raise RuntimeError("the model is already sharded (shard_model() runs once)")
        self.dp_shard_mesh = self.pconfig.device_mesh[Strategies.DP_SHARD.value]
        self.dp_shard_group = self.dp_shard_mesh.get_group()
        # host-resident shards cannot live in symmetric device memory
        self.coll = make_unit_collectives("nccl" if self.cpu_offload else self.collectives_kind, self.device,
                                          self.dp_shard_group)
        for buf in self.model.buffers():
            buf.data = buf.data.to(self.device)
        layers = get_fsdp_units(self.model)
        specs = []
        owned: set[int] = set()
        for i, sub in enumerate(layers):
            named = [(self.state_names[id(p)][0], p) for _, p in sub.named_parameters()]
            if owned.intersection(id(p) for _, p in named):
                raise ValueError("a parameter appears in two FSDP units; each parameter needs exactly one owner")
            if not named:
                continue
            owned.update(id(p) for _, p in named)
            ckpt = self.activation_checkpoint and (i % self.checkpoint_every_n == 0)
            for gi, group in enumerate(group_named_parameters(named)):
                specs.append((sub, group, ckpt and gi == 0, sub is not self.model, gi == 0))
        root_specs = []
        if layers != [self.model]:
            root = [(self.state_names[id(p)][0], p) for _, p in self.model.named_parameters()
                    if id(p) not in owned]
            if root:
                root_specs = [(self.model, g, False, False, False) for g in group_named_parameters(root)]
                owned.update(id(p) for _, p in root)
        if owned != {id(p) for p in self.model.parameters()}:
            raise RuntimeError("some model parameters ended up in no FSDP unit")
        all_specs = root_specs + specs
        for i, (sub, named, ckpt, reshard, primary) in enumerate(all_specs):
            unit = DPParamUnit(sub, self.dp_shard_mesh, i, self.coll, cpu_offload=self.cpu_offload,
                               use_activation_checkpoint=ckpt, device=self.device, named_parameters=named,
                               reshard_after_forward=reshard,
                               overlap_backward_reductions=self.overlap_backward_reductions)
            unit.shard()
            unit._layer_primary = primary
            self.units.append(unit)
        if hasattr(self.coll, "prepare"):
            self.coll.prepare(self.units)
        self.root_units = [u for u in self.units if u.module is self.model]
        for i, unit in enumerate(self.units):
            unit.next_fwd = self.units[i + 1] if i + 1 < len(self.units) else None
            unit.next_bwd = self.units[i - 1] if i > 0 else None
        # route every layer's forward through the unit function
        layer_units: dict[int, list[DPParamUnit]] = {}
        for u in self.units:
            if u.module is not self.model:
                layer_units.setdefault(id(u.module), []).append(u)
        for sub in layers:
            us = layer_units.get(id(sub))
            if not us:
                continue
            if len(us) != 1:
                raise NotImplementedError("Layers mixing parameter dtypes / frozen parameters are not supported")
            self._wrap_layer(sub, us[0])
        self._root_hook = self.model.register_forward_pre_hook(self._root_pre_forward)

    def _wrap_layer(self, layer: nn.Module, unit: DPParamUnit) -> None:
        orig = layer.forward
        self._orig_forwards[id(layer)] = orig
        wrapper = self

        def forward(x, *args):
            if not torch.is_grad_enabled():
                unit.all_gather()
                if unit.next_fwd is not None:
                    unit.next_fwd.prefetch()
                out = orig(x, *args)
                if unit.reshard_after_forward:
                    unit.free_full_params()
                return out
            y, *extras = _UnitFn.apply(wrapper, unit, orig, len(args), x, *args)
            sink = _sink_of(unit)
            if sink is not None:
                sink.extend(extras)
            return y

        layer.forward = forward

    def _deferred_root(self):
        """(root unit, embedding meta, embedding module, final norm module) when
        the root unit can be gathered in the background of the forward pass:
        one root unit on the NVLink data plane holding the token embedding, no
        tensor parallelism.  The embedding rows of the batch are then read
        straight from the owners' shards (the table is row-sharded exactly as
        a vocabulary-parallel embedding) and the full gather is waited for only
        before the final norm / LM head."""
        if getattr(self, "_deferred_root_info", 0) != 0:
            return self._deferred_root_info
        info = None
        inner = getattr(self.model, "model", None)
        emb = getattr(inner, "embed_tokens", None)
        norm = getattr(inner, "norm", None)
        ctx = getattr(self.model, "ctx", None)
        if (os.environ.get("PB_DEFER_ROOT_GATHER", "1") != "0"
                and len(self.root_units) == 1 and emb is not None and norm is not None and self.device.type == "cuda"
                and getattr(self.root_units[0], "_p2p", None) is not None and getattr(ctx, "tp_size", 1) == 1
                and getattr(self.coll, "name", "") == "p2p"):
            root = self.root_units[0]
            metas = [m for m in root.param_metas if m.parameter is emb.weight]
            if metas and metas[0].parameter.dtype == torch.bfloat16 and (metas[0].shape[1] * 2) % 16 == 0:
                info = (root, metas[0], emb, norm)
                self._norm_hook = norm.register_forward_pre_hook(lambda mod, args: root.wait_for_prefetch())
        self._deferred_root_info = info
        return info

    def _sharded_embedding_reader(self, root, meta):
        buf = root._p2p
        bases = [p + meta.bucket_offset * 2 for p in buf.peer_ptrs]
        pr, H = meta.padded_rows, meta.shape[1]

        def read(flat_ids):
            from ..ops._ext import ext

            rank = torch.div(flat_ids, pr, rounding_mode="floor")
            row = flat_ids - rank * pr
            out = torch.empty(flat_ids.numel(), H, device=flat_ids.device, dtype=torch.bfloat16)
            ext().row_gather(out, rank.to(torch.int32), row.contiguous(), bases, H * 2)
            return out

        return read

    def _root_pre_forward(self, module, args):
        begin = getattr(self.coll, "begin_forward", None) if self.coll is not None else None
        if begin is not None:
            begin()
        deferred = self._deferred_root()
        if deferred is not None:
            root, meta, emb, _ = deferred
            # every rank's shards are current (its optimizer step is done) ...
            root._p2p.barrier(0, self.coll.limit_s)
            self.coll._need_barrier = False
            # ... so the gather runs in the background and the batch's rows are
            # read from the shards directly
            root.prefetch()
            emb._sharded_lookup = self._sharded_embedding_reader(root, meta)
        else:
            for u in self.root_units:
                u.all_gather()
        nxt = self.root_units[-1].next_fwd if self.root_units else None
        if nxt is not None:
            nxt.prefetch()
        return None

    # ------------------------------------------------------------------ backward
    def prepare_backward(self, loss: torch.Tensor):
        if not self.is_active:
            return
        if not isinstance(loss, torch.Tensor):
            raise TypeError("prepare_backward() takes the loss tensor of the step")
        if self._backward_prepared:
            raise RuntimeError("prepare_backward() was called twice in one step")
        self._done_units.clear()
        self._deferred.clear()
        self._backward_prepared = True

    def _unit_backward_done(self, unit: DPParamUnit, grads: list) -> None:
        if not self._backward_prepared:
            raise RuntimeError("an FSDP unit finished its backward before prepare_backward() was called")
        self._done_units.add(unit.unit_index)
        missing = [m.name for m, g in zip(unit.param_metas, grads) if g is None]
        if missing and not self.find_unused_parameters:
            raise RuntimeError(
                f"FSDP backward ended before every expected parameter gradient was accumulated: "
                f"[{{'unit': {unit.unit_index}, 'missing_gradients': {missing}}}]")
        if self.overlap_backward_reductions and not self.find_unused_parameters:
            self._launch(unit, grads)
        else:
            self._deferred[unit.unit_index] = grads
        unit.free_full_params()

    def _launch(self, unit: DPParamUnit, grads: list) -> None:
        while len(self._inflight) >= self._max_inflight:
            self._inflight.pop(0).finish_gradient_reduction()
        unit.reduce_gradients(grads)
        self._inflight.append(unit)

    def finalize_backward(self):
        if not self.is_active:
            return
        if not self._backward_prepared:
            raise RuntimeError("finalize_backward() without prepare_backward() in this step")
        # root units: gradients arrived through autograd on the full params
        for u in self.root_units:
            grads = [m.parameter.grad for m in u.param_metas]
            for m in u.param_metas:
                m.parameter.grad = None
            if any(g is None for g in grads) and not self.find_unused_parameters and u.requires_grad:
                missing = [m.name for m, g in zip(u.param_metas, grads) if g is None]
                raise RuntimeError(
                    f"FSDP backward ended before every expected parameter gradient was accumulated: "
                    f"[{{'unit': {u.unit_index}, 'missing_gradients': {missing}}}]")
            if u.requires_grad:
                self._done_units.add(u.unit_index)
                if self.overlap_backward_reductions and not self.find_unused_parameters:
                    self._launch(u, grads)
                else:
                    self._deferred[u.unit_index] = grads
        trainable = [u for u in self.units if u.requires_grad]
        if not self.find_unused_parameters:
            pending = [u.unit_index for u in trainable if u.unit_index not in self._done_units]
            if pending:
                raise RuntimeError(f"FSDP backward ended before every expected parameter gradient was "
                                   f"accumulated: units {pending} never ran backward")
            if not self.overlap_backward_reductions:
                for u in reversed(trainable):
                    self._launch(u, self._deferred.pop(u.unit_index))
        else:
            # fixed reverse order on every rank; zeros where nothing ran locally
            for u in reversed(trainable):
                grads = self._deferred.pop(u.unit_index, [None] * len(u.param_metas))
                self._launch(u, grads)
        for u in self._inflight:
            u.finish_gradient_reduction()
        self._inflight.clear()
        participation = None
        if self.find_unused_parameters:
            bits = torch.tensor([int(p) for u in trainable for p in u._participation], dtype=torch.int32,
                                device=self.device)
            if bits.numel():
                dist.all_reduce(bits, op=dist.ReduceOp.SUM, group=self.dp_shard_group)
            flags = bits.gt(0).tolist()
            participation, k = {}, 0
            for u in trainable:
                participation[u.unit_index] = flags[k:k + len(u.param_metas)]
                k += len(u.param_metas)
        for u in trainable:
            u.attach_gradients(None if participation is None else participation[u.unit_index])
        for u in self.units:
            u.free_full_params()
        self._backward_prepared = False
        self._done_units.clear()

    def zero_grad(self) -> None:
        for u in self.units:
            u.zero_grad()

    def stage_offloaded_gradients(self) -> None:
        """cpu_offload: bring the reduced gradients to the host shards (no-op otherwise)."""
        if self.cpu_offload:
            for u in self.units:
                u.stage_offloaded_gradients()

    # ------------------------------------------------------------------ params
    def get_optimizer_params(self) -> list[nn.Parameter]:
        if not self.units:
            return [p for p in self.model.parameters() if p.requires_grad]
        return [m.sharded_param for u in self.units if u.requires_grad for m in u.param_metas]

    def get_sharded_params(self) -> list[nn.Parameter]:
        return [m.sharded_param for u in self.units for m in u.param_metas]

    def grad_buckets(self) -> list[torch.Tensor]:
        """Reduced gradient shard buckets (one flat tensor per unit)."""
        return [u.grad_shards() for u in self.units if u.requires_grad and u.grad_shards() is not None]

    def clip_grad_norm_(self, max_norm: float) -> torch.Tensor:
        """Clip by one norm shared by the shard group (no host synchronisation)."""
        params = self.get_optimizer_params()
        if not self.is_active:
            return torch.nn.utils.clip_grad_norm_(params, max_norm)
        sq = torch.zeros((), dtype=torch.float32, device=self.device)
        for p in params:
            if p.grad is not None:
                sq += local_tensor(p.grad).detach().float().pow(2).sum().to(self.device)
        dist.all_reduce(sq, op=dist.ReduceOp.SUM, group=self.dp_shard_group)
        total = sq.sqrt()
        coef = (max_norm / (total + 1e-6)).clamp(max=1.0)
        for p in params:
            if p.grad is not None:
                g = local_tensor(p.grad)
                g.mul_(coef.to(g.device, g.dtype))
        return total

    @property
    def is_active(self) -> bool:
        return len(self.units) > 0

    def remove_hooks(self):
        for u in self.units:
            u.all_gather()
        for layer in get_fsdp_units(self.model):
            if id(layer) in self._orig_forwards:
                layer.forward = self._orig_forwards.pop(id(layer))
        if self._root_hook is not None:
            self._root_hook.remove()
            self._root_hook = None
        if getattr(self, "_norm_hook", None) is not None:
            self._norm_hook.remove()
            self._norm_hook = None
        self._deferred_root_info = 0
