"""ParallelEngine: forward / backward / optimizer step over MP and FSDP.

Same public surface as the reference engine (parallel/parallel/engine/
engine.py:20-324): ``forward(x, y)``, ``backward(loss)``, ``step()``,
``reduce_loss``, ``token_loss``, ``sync_buffers``, (sharded) state dicts,
``save/load_checkpoint``, ``save/load_full_model``, ``step_memory_stats``,
``lr``.  Composition order is the same: model-parallel wrapper first, then
FSDP over the model-parallel-local parameters, then AdamW over the shards.

Step differences (B200-first, same math):
* the global gradient norm, the clip coefficient and the non-finite flag are
  computed on the device in one multi-tensor pass and handed to the fused
  AdamW kernel (no per-parameter ``.item()`` syncs); a non-finite step
  leaves the parameters untouched and raises ``FloatingPointError`` on the
  next ``step()`` call (or immediately with ``sync_finite_check=True``);
* DP-replicate gradient averaging is one all-reduce per gradient bucket.
"""
from __future__ import annotations

import torch
import torch.distributed as dist

from ..profiling import (collective_phase, configure_collective_profiling, finish_collective_profile_step,
                         start_collective_profile_step, collective_profile)
from ..state import Strategies
from ..utils import DTYPE_DICT
from ..ops._ext import ext
from .checkpoint import CheckpointManager
from .fsdp import FSDPWrapper
from .fsdp_utils import local_tensor
from .model_parallel import ModelParallelWrapper
from .optim import FusedAdamW


def _cfg_get(node, key, default):
    try:
        return node.get(key, default)
    except AttributeError:
        return getattr(node, key, default)


class ParallelEngine:
    def __init__(self, model, tokenizer, pconfig, cfg, device, mp_plan=None):
        self.tokenizer = tokenizer
        self.pconfig = pconfig
        self.cfg = cfg
        self.device = device
        self.use_amp = cfg.config.use_amp
        if self.use_amp and cfg.config.amp_dtype not in ("bf16", "fp16"):
            raise ValueError("config.amp_dtype has to be 'bf16' or 'fp16' when config.use_amp is set")
        self.amp_dtype = DTYPE_DICT.get(cfg.config.amp_dtype, torch.float32)
        self.grad_scaler = torch.amp.GradScaler(pconfig.device_type or device.type,
                                                enabled=self.use_amp and self.amp_dtype == torch.float16)
        eng = cfg.engine
        self.mp_wrapper = ModelParallelWrapper(model, pconfig, device=device, plan=mp_plan,
                                               collectives=_cfg_get(eng, "collectives", "auto"))
        self.fsdp_wrapper = FSDPWrapper(
            model, pconfig, cpu_offload=eng.cpu_offload, activation_checkpoint=eng.activation_checkpoint,
            checkpoint_every_n=eng.checkpoint_every_n,
            find_unused_parameters=_cfg_get(eng, "find_unused_parameters", False),
            overlap_backward_reductions=_cfg_get(eng, "overlap_backward_reductions", True), device=device,
            collectives=_cfg_get(eng, "collectives", "auto"))
        self.fsdp_wrapper.shard_model()
        self.mp_wrapper.attach_fsdp(self.fsdp_wrapper)
        self.model = model
        self.optimizer_params = self.fsdp_wrapper.get_optimizer_params()
        self._sync_initial_state()
        self.optimizer = FusedAdamW(self.optimizer_params, lr=cfg.model.learning_rate,
                                    betas=(cfg.optim.adam_beta1, cfg.optim.adam_beta2),
                                    weight_decay=cfg.optim.weight_decay,
                                    state_dtype=_cfg_get(eng, "optimizer_state_dtype", "param"))
        self.optimizer.zero_grad(set_to_none=True)
        self.checkpoint = CheckpointManager(self)
        configure_collective_profiling(enabled=_cfg_get(eng, "collective_profiling", False), device=device)
        self.sync_finite_check = bool(_cfg_get(eng, "sync_finite_check", False))
        self._pending_nonfinite: torch.Tensor | None = None
        # asynchronous read-back of the non-finite flag: copied into pinned
        # host memory behind an event at the end of step k, read at step k+1
        self._flag_host: torch.Tensor | None = None
        self._err_host: torch.Tensor | None = None
        self._flag_event = None
        self._last_grad_norm: torch.Tensor | None = None
        self._graph = None
        self._graph_pending = None
        self._captured_flag: torch.Tensor | None = None
        self.reset_step_memory_stats()

    # ------------------------------------------------------------------ init
    def _sync_initial_state(self):
        """Every data-parallel replica starts from identical state."""
        if self.pconfig.device_mesh is None:
            return
        for dim in (Strategies.DP_REPLICATE, Strategies.DP_SHARD):
            group = self.pconfig.group(dim)
            if group is None:
                continue
            src = dist.get_global_rank(group, 0)
            tensors = list(self.model.buffers())
            if not self.fsdp_wrapper.is_active:
                tensors += list(self.model.parameters())
            elif dim == Strategies.DP_REPLICATE:
                tensors += self.fsdp_wrapper.get_sharded_params()
            for t in tensors:
                v = local_tensor(t).detach()
                if v.device.type == self.device.type:
                    dist.broadcast(v, src=src, group=group)
                else:
                    staged = v.to(self.device)
                    dist.broadcast(staged, src=src, group=group)
                    v.copy_(staged.to(v.device))

    @property
    def lr(self):
        return self.optimizer.param_groups[0]["lr"]

    # ------------------------------------------------------------------ memory
    def reset_step_memory_stats(self):
        self._forward_peak_memory_allocated = 0
        self._backward_peak_memory_allocated = 0
        start_collective_profile_step()

    def finish_step_collective_profile(self) -> list[str]:
        return finish_collective_profile_step()

    def _reset_peak(self):
        if self.device.type == "cuda":
            torch.cuda.reset_peak_memory_stats(self.device)

    def _peak(self) -> int:
        return torch.cuda.max_memory_allocated(self.device) if self.device.type == "cuda" else 0

    def step_memory_stats(self) -> dict[str, int]:
        peaks = torch.tensor([self._forward_peak_memory_allocated, self._backward_peak_memory_allocated],
                             dtype=torch.int64, device=self.device)
        if dist.is_initialized():
            dist.all_reduce(peaks, op=dist.ReduceOp.MAX)
        return {"forward_peak_allocated_bytes": int(peaks[0].item()),
                "backward_peak_allocated_bytes": int(peaks[1].item())}

    # ------------------------------------------------------------------ fwd / bwd
    def forward(self, x, y):
        self._reset_peak()
        with collective_phase("forward"):
            with torch.autocast(device_type=self.device.type, dtype=self.amp_dtype,
                                enabled=self.use_amp and self.device.type == "cuda"):
                if self.mp_wrapper.is_active:
                    outputs = self.model(input_ids=x)
                    outputs.loss = self.mp_wrapper.training_loss(outputs, y)
                else:
                    outputs = self.model(input_ids=x, labels=y)
        self._forward_peak_memory_allocated = max(self._forward_peak_memory_allocated, self._peak())
        return outputs

    def sync_buffers(self):
        """Broadcast every buffer from the first replica / shard rank."""
        if self.pconfig.device_mesh is None:
            return
        bufs = list(self.model.buffers())
        for dim in (Strategies.DP_REPLICATE, Strategies.DP_SHARD):
            group = self.pconfig.group(dim)
            if group is None:
                continue
            src = dist.get_global_rank(group, 0)
            for b in bufs:
                dist.broadcast(b, src=src, group=group)

    def backward(self, loss):
        self._reset_peak()
        with collective_phase("backward"):
            self.fsdp_wrapper.prepare_backward(loss)
            with self.mp_wrapper.backward_context():
                if self.grad_scaler.is_enabled():
                    self.grad_scaler.scale(loss).backward()
                else:
                    loss.backward()
            self.fsdp_wrapper.finalize_backward()
        self._backward_peak_memory_allocated = max(self._backward_peak_memory_allocated, self._peak())

    # ------------------------------------------------------------------ step
    def step(self):
        with collective_phase("optimizer"):
            self._step_impl()

    # ------------------------------------------------------------------ whole step
    def train_step(self, x, y):
        """Forward, backward and optimizer step on one batch; returns the loss
        as a device tensor (no host synchronisation).  ``x`` / ``y`` are token
        ids [B, S], or [A, B, S] for A micro-batches accumulated into one
        optimizer step (each micro-batch loss scaled by 1/A, as the training
        loop does with ``config.grad_accum_steps``; the returned loss is their
        sum).  After ``capture_train_step`` this replays the captured CUDA
        graph instead (the returned tensor is then the graph's static loss,
        overwritten by the next call)."""
        if self._graph is not None:
            return self._graph.replay(x, y)
        if self._graph_pending is not None:
            return self._pending_graph_step(x, y)
        return self._eager_step(x, y)

    def _eager_step(self, x, y):
        if x.dim() == 2:
            outputs = self.forward(x, y)
            self.backward(outputs.loss)
            self.step()
            return outputs.loss.detach()
        A = x.shape[0]
        total = None
        for a in range(A):
            loss = self.forward(x[a], y[a]).loss / A
            self.backward(loss)
            total = loss.detach() if total is None else total + loss.detach()
        self.step()
        return total

    def enable_graph_capture(self, warmup_steps: int = 2):
        """From the next ``train_step`` on: run ``warmup_steps`` ordinary steps
        (each on its own batch) on the capture stream, then capture the step
        at the following call and replay it from then on.  Unlike
        ``capture_train_step`` no batch is trained on more than once, so a
        training run's trajectory is the eager one.  This is what
        ``engine.compile=true`` selects: the reference compiles the model with
        ``torch.compile`` there (parallel/parallel/train.py:60-66); here the
        kernels are already hand-written and the remaining cost is launch
        overhead, which the graph removes."""
        from .graph_step import capture_unsupported

        why = capture_unsupported(self)
        if why is not None:
            raise NotImplementedError(f"engine.compile (CUDA-graph step) does not support {why}")
        if self.device.type != "cuda":
            raise NotImplementedError("engine.compile captures the training step as a CUDA graph; it needs a "
                                      "CUDA device")
        if warmup_steps < 1:
            raise ValueError("at least one eager step must run on the capture stream before the capture")
        self._graph = None
        self._graph_pending = {"stream": torch.cuda.Stream(device=self.device), "left": int(warmup_steps)}

    def _pending_graph_step(self, x, y):
        from .graph_step import GraphedTrainStep

        st = self._graph_pending
        cur = torch.cuda.current_stream(self.device)
        if st["left"] > 0:
            st["left"] -= 1
            st["stream"].wait_stream(cur)
            with torch.cuda.stream(st["stream"]):
                loss = self._eager_step(x, y)
            cur.wait_stream(st["stream"])
            loss.record_stream(cur)
            return loss
        self._graph_pending = None
        self._graph = GraphedTrainStep(self, x, y, warmup=0, stream=st["stream"])
        return self._graph.replay(x, y)

    def capture_train_step(self, x, y, warmup: int = 3):
        """Run ``warmup`` eager steps on (x, y) (they train on it), then capture
        one whole training step - forward, backward, reductions, optimizer - as
        a CUDA graph that ``train_step`` replays from then on.  Every rank must
        call this at the same point.  See ``parallel_b200/parallel/graph_step.py``."""
        from .graph_step import GraphedTrainStep

        self._graph = self._graph_pending = None
        self._graph = GraphedTrainStep(self, x, y, warmup=warmup)
        return self._graph

    def release_graph(self):
        """Drop the captured step (call before destroying the process group)."""
        if self._graph is not None:
            self._graph.release()
        self._graph = self._graph_pending = None

    def _check_pending_nonfinite(self):
        if self._pending_nonfinite is None:
            return
        err = 0
        if self._flag_event is not None:
            # waits only for the end of the previous optimizer step, which the
            # GPU has normally passed long ago (no pipeline drain)
            self._flag_event.synchronize()
            bad = bool(self._flag_host[0].item())
            err = int(self._err_host[0]) if self._err_host is not None else 0
            self._flag_event = None
        else:
            bad = bool(self._pending_nonfinite.item())
        self._pending_nonfinite = None
        if err:
            # a bounded device wait gave up during that step (its results are not
            # trustworthy): clear the word and fail on every rank that saw it
            from ..ops._ext import clear_device_errors
            from .comm.p2p import CollectiveTimeout

            clear_device_errors(self.device.index)
            msg = f"device error code {err} during the previous step (1 = pipeline wait, 2 = peer wait timeout)"
            raise CollectiveTimeout(msg) if err == 2 else RuntimeError(msg)
        if bad:
            raise FloatingPointError("gradient norm is not finite (inf or nan in some gradient); step skipped")

    def _defer_nonfinite_check(self, flag: torch.Tensor):
        self._pending_nonfinite = flag
        if flag.is_cuda:
            if self._flag_host is None:
                self._flag_host = torch.zeros(1, dtype=flag.dtype, pin_memory=True)
                self._err_host = torch.zeros(1, dtype=torch.int32, pin_memory=True)
            self._flag_host.copy_(flag.reshape(1), non_blocking=True)
            # the device error word (bounded waits that timed out) travels with the flag
            ext().error_word_copy_async(self._err_host)
            self._flag_event = torch.cuda.Event()
            self._flag_event.record()

    def _grad_lists(self):
        """(grad tensors, weights) for the norm: replicated TP params count once."""
        grads, weights = [], []
        rep_weight = self.mp_wrapper.replicated_grad_weight()
        for p in self.optimizer_params:
            if p.grad is None:
                continue
            g = local_tensor(p.grad)
            w = rep_weight if self.mp_wrapper.is_replicated_param(p) else 1.0
            grads.append(g)
            weights.append(w)
        return grads, weights

    def _norm_groups(self):
        groups = []
        if self.mp_wrapper.is_active:
            g = self.pconfig.group(Strategies.TP)
            if g is not None:
                groups.append(g)
        if self.fsdp_wrapper.is_active:
            groups.append(self.fsdp_wrapper.dp_shard_group)
        return groups

    def _step_impl(self):
        capturing = self.device.type == "cuda" and torch.cuda.is_current_stream_capturing()
        if not capturing:
            try:
                self._check_pending_nonfinite()
            except (FloatingPointError, RuntimeError):
                # the previous step failed (reported one step late): this step is
                # abandoned too, like the synchronous check's failing step
                self.optimizer.zero_grad(set_to_none=True)
                self.fsdp_wrapper.zero_grad()
                raise
        self._average_gradients()
        self.fsdp_wrapper.stage_offloaded_gradients()
        if self.grad_scaler.is_enabled():
            self.grad_scaler.unscale_(self.optimizer)
        cuda = self.device.type == "cuda" and all(local_tensor(p).is_cuda for p in self.optimizer_params)
        max_norm = float(self.cfg.model.clip_grad_norm)
        if cuda and not self.grad_scaler.is_enabled():
            grads, weights = self._grad_lists()
            sq = torch.empty(1, dtype=torch.float32, device=self.device)
            flag = torch.empty(1, dtype=torch.int32, device=self.device)
            by_dtype: dict = {}
            for g, w in zip(grads, weights):
                by_dtype.setdefault(g.dtype, ([], []))
                by_dtype[g.dtype][0].append(g if g.is_contiguous() else g.contiguous())
                by_dtype[g.dtype][1].append(w)
            if not by_dtype:
                sq.zero_()
                flag.zero_()
            # per-chunk partials summed in chunk order: the norm is reproducible
            for i, (gs, ws) in enumerate(by_dtype.values()):
                ext().sumsq(gs, ws, sq, flag, i > 0)
            sq, flag = self._reduce_norm_and_flag(sq, flag)
            scale = None
            if max_norm > 0.0:
                scale = torch.empty(1, dtype=torch.float32, device=self.device)
                ext().clip_coef(sq, max_norm, scale)
            self._last_grad_norm = sq.sqrt()
            self.optimizer.step(grad_scale=scale, skip=flag)
            self.optimizer.zero_grad(set_to_none=True)
            self.fsdp_wrapper.zero_grad()
            if capturing:  # read back after each replay by the graph runner
                self._captured_flag = flag
            elif self.sync_finite_check:
                self._pending_nonfinite = flag
                self._check_pending_nonfinite()
            else:
                self._defer_nonfinite_check(flag)
            return
        if capturing:
            raise RuntimeError("Only the CUDA step without a gradient scaler can be captured in a CUDA graph")
        # generic path (CPU / fp16 scaler): reference semantics with host syncs
        finite = self._grads_are_finite()
        if finite and max_norm > 0.0:
            if self.mp_wrapper.is_active:
                self._last_grad_norm = self.mp_wrapper.clip_grad_norm_(self.optimizer_params, max_norm)
            else:
                self._last_grad_norm = self.fsdp_wrapper.clip_grad_norm_(max_norm)
        if not finite:
            if not self.grad_scaler.is_enabled():
                self.optimizer.zero_grad(set_to_none=True)
                self.fsdp_wrapper.zero_grad()
                raise FloatingPointError("gradient norm is not finite (inf or nan in some gradient); step skipped")
            self.grad_scaler.update(new_scale=self.grad_scaler.get_scale() / 2.0)
        else:
            if self.grad_scaler.is_enabled():
                self.grad_scaler.step(self.optimizer)
                self.grad_scaler.update()
            else:
                self.optimizer.step()
        self.optimizer.zero_grad(set_to_none=True)
        self.fsdp_wrapper.zero_grad()

    def _reduce_norm_and_flag(self, sq: torch.Tensor, flag: torch.Tensor):
        """Sum the squared-gradient partial over the norm groups (TP, then the
        shard group) and the non-finite flag over every data / model group.
        On CUDA with NVLink peer access both travel in one peer-memory kernel
        per group ([sq, flag] summed; flag > 0 means non-finite anywhere);
        otherwise NCCL all-reduces (SUM, MAX)."""
        norm_groups = self._norm_groups()
        flag_groups = [g for dim in (Strategies.DP_REPLICATE, Strategies.TP, Strategies.DP_SHARD)
                       if (g := self.pconfig.group(dim)) is not None]
        groups = []
        for g in norm_groups + flag_groups:
            if all(g is not h for h in groups) and dist.get_world_size(g) > 1:
                groups.append(g)
        small = None
        if groups and self.device.type == "cuda" and _cfg_get(self.cfg.engine, "collectives", "auto") != "nccl":
            from .comm.p2p import P2PSmallAllReduce

            small = [P2PSmallAllReduce.get(g, self.device) for g in groups]
            if any(x is None for x in small):
                small = None
        if small is None:
            for group in norm_groups:
                dist.all_reduce(sq, op=dist.ReduceOp.SUM, group=group)
            for group in flag_groups:
                dist.all_reduce(flag, op=dist.ReduceOp.MAX, group=group)
            return sq, flag
        packed = torch.cat([sq.reshape(1), flag.reshape(1).to(torch.float32)])
        for g, ar in zip(groups, small):
            if any(g is h for h in norm_groups):
                ar.all_reduce_(packed, "sum")
            else:  # replicas hold the same gradients: only the flag is combined
                ar.all_reduce_(packed[1:], "sum")
        return packed[:1], (packed[1:] > 0).to(torch.int32)

    def _replica_mean(self, tensors, group, op: str) -> None:
        """Mean over the replicate group: NVLink peer memory when the buffers
        qualify (``ReplicaMeanAllReduce``), else one NCCL / gloo all-reduce each."""
        if not tensors:
            return
        peer = None
        if _cfg_get(self.cfg.engine, "collectives", "auto") != "nccl":
            from .comm.p2p import ReplicaMeanAllReduce

            peer = ReplicaMeanAllReduce.get(group, self.device, tensors)
        if peer is not None:
            with collective_profile(op, payload_bytes=sum(2 * t.numel() for t in tensors),
                                    mode="nvls" if peer.nvls is not None else "p2p", detail="replicate"):
                peer.mean_(tensors)
            return
        for t in tensors:
            with collective_profile(op, value=t, mode="replicate"):
                dist.all_reduce(t, op=dist.ReduceOp.SUM, group=group)
            t.div_(self.pconfig.dp_replicate_size)

    def _average_gradients(self):
        """Mean of the gradients over the replicate group."""
        if self.pconfig.dp_replicate_size <= 1 or self.pconfig.device_mesh is None:
            return
        group = self.pconfig.group(Strategies.DP_REPLICATE)
        if self.fsdp_wrapper.is_active:
            self._replica_mean(self.fsdp_wrapper.grad_buckets(), group, "fsdp_all_reduce")
            return
        # one participation bitmap for all parameters instead of the reference's
        # per-parameter flag and sync (parallel/parallel/engine/engine.py:224-247);
        # replicas without a local gradient contribute zeros, globally unused
        # parameters keep grad=None.  The bitmap is read on the host only by a
        # rank that lacks a local gradient: where every local gradient exists,
        # every parameter is used somewhere.
        params = list(self.optimizer_params)
        local = [p.grad is not None for p in params]
        has = torch.tensor([int(x) for x in local], dtype=torch.int32, device=self.device)
        if has.numel():
            dist.all_reduce(has, op=dist.ReduceOp.MAX, group=group)
        used = local if all(local) else has.tolist()
        grads = []
        for p, u in zip(params, used):
            if not u:
                p.grad = None
                continue
            if p.grad is None:
                p.grad = torch.zeros_like(p)
            grads.append(local_tensor(p.grad))
        self._replica_mean(grads, group, "dp_all_reduce")

    def _grads_are_finite(self) -> bool:
        finite = torch.ones((), dtype=torch.int32, device=self.device)
        for p in self.optimizer_params:
            g = p.grad
            if g is None:
                continue
            if not torch.isfinite(local_tensor(g)).all():
                finite.zero_()
                break
        if self.pconfig.device_mesh is not None:
            for dim in (Strategies.DP_REPLICATE, Strategies.TP, Strategies.DP_SHARD):
                group = self.pconfig.group(dim)
                if group is not None:
                    dist.all_reduce(finite, op=dist.ReduceOp.MIN, group=group)
        return bool(finite.item())

    @property
    def last_grad_norm(self):
        return self._last_grad_norm

    # ------------------------------------------------------------------ checkpoint facade
    def state_dict(self):
        return self.checkpoint.full_state_dict()

    def load_state_dict(self, state_dict, strict: bool = True):
        return self.checkpoint.load_full_state_dict(state_dict, strict=strict)

    def sharded_state_dict(self):
        return self.checkpoint.sharded_state_dict()

    def load_sharded_state_dict(self, state_dict, strict: bool = True):
        return self.checkpoint.load_sharded_state_dict(state_dict, strict=strict)

    def save_checkpoint(self, path, *, step: int, dataloader_state=None, eval_dataloader_state=None, metadata=None):
        return self.checkpoint.save(path, step=step, dataloader_state=dataloader_state,
                                    eval_dataloader_state=eval_dataloader_state, metadata=metadata)

    def load_checkpoint(self, path, *, strict: bool = True):
        return self.checkpoint.load(path, strict=strict)

    def save_full_model(self, path):
        return self.checkpoint.save_full_model(path)

    def load_full_model(self, path, *, strict: bool = True):
        return self.checkpoint.load_full_model(path, strict=strict)

    # ------------------------------------------------------------------ losses
    def reduce_loss(self, loss):
        out = loss.detach().float().clone()
        if not self.pconfig.dp_enabled or self.pconfig.device_mesh is None:
            return out
        for dim in (Strategies.DP_REPLICATE, Strategies.DP_SHARD):
            group = self.pconfig.group(dim)
            if group is None:
                continue
            dist.all_reduce(out, op=dist.ReduceOp.SUM, group=group)
            out.div_(dist.get_world_size(group))
        return out

    def token_loss(self, logits, labels, reduction: str = "mean"):
        return self.mp_wrapper.token_loss(logits, labels, reduction=reduction)
