"""A whole training step captured as one CUDA graph and replayed.

At the benchmark shapes (Qwen3-0.6B, 8,192 tokens per GPU) a step issues
about 1,100 kernels (1,700 with FSDP activation checkpointing), each behind
a Python autograd Function, tensor-map encodes and allocator calls; with
FSDP units the host falls behind the GPU in the backward.  Capturing the
forward, the backward (with the FSDP gathers and reductions on their side
streams), the gradient norm and the optimizer into one graph turns a step
into one ``cudaGraphLaunch``.  The reference has no counterpart (it runs
eagerly, parallel/parallel/train.py:120-160); the step's semantics are
unchanged.

What makes the step replayable:

* the batch is copied into input buffers owned by the runner;
* the memory of the step comes from the graph's private pool, so every
  activation, gathered unit and gradient has the same address at every
  replay, and the TMA descriptors encoded at capture time stay valid;
* the peer-memory barriers count epochs on the device
  (``SymmBuffer.epochs``);
* AdamW reads lr and the bias corrections from a device tensor that the
  host refreshes before each replay (``FusedAdamW.advance_graph_step``),
  so learning-rate schedules keep working;
* the non-finite flag of a replay is read back asynchronously and checked
  at the next replay, as in eager steps.

Cross-replay safety of the symmetric staging buffers: a replay's first
reuse of a reduce-scatter slot or of a shard comes after the previous
step's gradient-norm all-reduce, which no rank passes before every rank's
reductions and gathers of that step have finished.

MoE layers are capturable: their routing plan, expert GEMM tile counts and
exchange sizes live on the device (``ops.moe.routed_experts``).

Model parallelism is capturable too: the NVLink kernels of TP / SP / EP wait
on device epochs and per-call counters that are reset on the stream.

Not capturable (the runner refuses them, ``capture_unsupported``): expert
parallelism on NCCL all-to-alls (host-read split sizes), fp16 loss scaling (host decisions), CPU offload
(host optimizer), usage bitmaps read on the host (FSDP with
find_unused_parameters, DP-replicate without FSDP), CPU devices.
"""
from __future__ import annotations

import torch
import torch.distributed as dist


def capture_unsupported(engine) -> str | None:
    """Why the engine's training step cannot be captured (each of these makes
    a host decision or a host read inside the step), or None."""
    fsdp = engine.fsdp_wrapper
    cfg = getattr(engine.model, "config", None)
    if getattr(cfg, "is_moe", False) and not (1 <= cfg.num_experts <= 256 and cfg.hidden_size % 8 == 0):
        return "MoE models whose routing cannot run on the device (more than 256 experts)"
    runtime = getattr(engine.mp_wrapper, "expert_runtime", None) if engine.mp_wrapper.is_active else None
    if runtime is not None and getattr(runtime, "dispatcher", None) is not None \
            and getattr(runtime, "transport", "local") is None:
        return "expert parallelism on NCCL all-to-alls (their split sizes are read on the host)"
    if engine.grad_scaler.is_enabled():
        return "fp16 loss scaling (its skip / rescale decisions are taken on the host)"
    if fsdp.is_active and fsdp.cpu_offload:
        return "engine.cpu_offload (the optimizer steps on host memory)"
    if fsdp.is_active and fsdp.find_unused_parameters:
        return "engine.find_unused_parameters (the usage bitmap is read on the host)"
    if not fsdp.is_active and engine.pconfig.dp_replicate_size > 1:
        return "DP-replicate without FSDP (the gradient participation bitmap is read on the host)"
    if not hasattr(engine.optimizer, "enable_graph_hyper"):
        return "optimizers other than FusedAdamW"
    return None


class GraphedTrainStep:
    def __init__(self, engine, x: torch.Tensor, y: torch.Tensor, warmup: int = 3, stream=None):
        """``warmup`` eager steps on (x, y) run on the capture stream first.  With
        ``warmup=0`` the caller passes the ``stream`` on which its own eager
        steps already ran (``ParallelEngine.enable_graph_capture``)."""
        if engine.device.type != "cuda":
            raise RuntimeError("CUDA-graph steps need a CUDA device")
        why = capture_unsupported(engine)
        if why is not None:
            raise NotImplementedError(f"CUDA-graph steps do not support {why}")
        self.engine = engine
        dev = engine.device
        self.x = torch.empty(x.shape, dtype=x.dtype, device=dev)
        self.y = torch.empty(y.shape, dtype=y.dtype, device=dev)
        self.x.copy_(x)
        self.y.copy_(y)
        # warm-up on the stream the capture will use: lazy initialisation of
        # optimizer state, kernel attributes, NCCL communicators and symmetric
        # buffers happens here, outside the capture
        if warmup < 1 and stream is None:
            raise ValueError("warmup=0 needs the stream on which the eager warm-up steps ran")
        self.stream = stream if stream is not None else torch.cuda.Stream(device=dev)
        self.stream.wait_stream(torch.cuda.current_stream(dev))
        with torch.cuda.stream(self.stream):
            for _ in range(warmup):
                engine.train_step(self.x, self.y)
        torch.cuda.current_stream(dev).wait_stream(self.stream)
        torch.cuda.synchronize(dev)
        engine._check_pending_nonfinite()
        if dist.is_initialized():
            dist.barrier()
            torch.cuda.synchronize(dev)
        coll = getattr(engine.fsdp_wrapper, "coll", None)
        if coll is not None and hasattr(coll, "reset_step_events"):
            coll.reset_step_events()
        opt = engine.optimizer
        opt.enable_graph_hyper(dev)
        counts = opt.graph_step_counts()
        self.graph = torch.cuda.CUDAGraph()
        try:
            with torch.cuda.graph(self.graph, stream=self.stream):
                self.loss = engine.train_step(self.x, self.y)
        finally:
            # the capture advanced the host step counters without running
            opt.restore_step_counts(counts)
        self.flag = engine._captured_flag
        engine._captured_flag = None
        if self.flag is None:
            raise RuntimeError("the captured step produced no non-finite flag")
        if coll is not None and hasattr(coll, "reset_step_events"):
            coll.reset_step_events()
        torch.cuda.synchronize(dev)

    def replay(self, x: torch.Tensor, y: torch.Tensor) -> torch.Tensor:
        eng = self.engine
        eng._check_pending_nonfinite()
        if x.shape != self.x.shape or y.shape != self.y.shape:
            raise ValueError(f"captured for batches of {tuple(self.x.shape)}, got {tuple(x.shape)}")
        if x.data_ptr() != self.x.data_ptr():
            self.x.copy_(x, non_blocking=True)
        if y.data_ptr() != self.y.data_ptr():
            self.y.copy_(y, non_blocking=True)
        eng.optimizer.advance_graph_step()
        self.graph.replay()
        eng._defer_nonfinite_check(self.flag)
        return self.loss

    def release(self) -> None:
        self.graph.reset()
        self.loss = self.flag = None
