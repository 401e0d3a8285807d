"""Training entry point.

    torchrun --standalone --nproc-per-node N -m parallel_b200.train [override.yaml] key=value ...

Same flow and overrides as the reference trainer (parallel/parallel/
train.py:23-197): config -> process group -> mesh -> RNG policy -> model ->
engine -> (resume) -> loaders -> loop of grad-accumulation micro-batches,
optimizer step, logging (loss / lr / tok/s / forward and backward peak
memory, optional [COLLECTIVE] lines), periodic bits-per-byte eval and
sharded checkpoints.  ``data.synthetic=true`` trains on uniform random token
ids (no tokenizer or parquet files needed).  Throughput is also reported as
device-timed tokens/s (CUDA events, max over ranks).
"""
from __future__ import annotations

import os
import time
from pathlib import Path

import torch
import torch.distributed as dist

from .config import load_cfg
from .dataloader import dist_data_loader, synthetic_data_loader
from .eval import eval_bpb, get_token_bytes
from .logging import configure_logging, get_logger
from .models.loading import load_causal_lm
from .parallel.engine import ParallelEngine
from .profiling import scheduled_torch_profiler
from .state import ParallelConfig, RuntimeState, init_dist
from .tracking import WandBTracker
from .utils import dist_cleanup

logger = get_logger(__name__)


def _load_dotenv():
    path = Path(".env")
    if not path.is_file():
        return
    for line in path.read_text().splitlines():
        line = line.strip()
        if line and not line.startswith("#") and "=" in line:
            k, v = line.split("=", 1)
            os.environ.setdefault(k.strip(), v.strip().strip('"').strip("'"))


def main(argv=None):
    _load_dotenv()
    cfg = load_cfg(argv=argv)
    RuntimeState(backend=cfg.config.backend)
    init_dist(cfg)
    configure_logging()
    pconfig = ParallelConfig(cfg)
    pconfig.set_device_mesh(cfg.config.device_type)
    device = pconfig.device
    wandb = WandBTracker(rank=pconfig.rank, enabled=os.environ.get("WANDB_MODE") != "disabled"
                         and bool(os.environ.get("WANDB_API_KEY")))
    wandb.start()
    wandb.store_init_config(cfg.to_container())
    seed = cfg.get("seed", 42)
    pconfig.model_init_rngs(seed=seed)
    model, mp_plan = load_causal_lm(cfg, pconfig)
    synthetic = bool(cfg.data.get("synthetic", False))
    tokenizer, token_bytes = None, None
    if not synthetic:
        from transformers import AutoTokenizer

        tokenizer = AutoTokenizer.from_pretrained(cfg.model.name)
        logger.info("Measuring the byte length of every token for bits-per-byte...")
        token_bytes = get_token_bytes(tokenizer)
    pconfig.model_train_rngs(seed=seed)
    # engine.compile: the whole training step is captured as a CUDA graph
    # (ParallelEngine.enable_graph_capture) - FSDP, DP-replicate and model
    # parallelism on the NVLink data plane included, which the reference's
    # torch.compile path refuses (train.py:45-66); enable_graph_capture names
    # anything that cannot be captured
    graph_step = bool(cfg.engine.compile)
    if graph_step and cfg.engine.get("collective_profiling", False):
        raise NotImplementedError("engine.compile replays the step as one graph; per-collective profiling needs "
                                  "eager steps")
    if pconfig.dp_shard_size <= 1 and not pconfig.model_parallel_enabled:
        model.to(device)
        model._layout_fused_weights()
    elif pconfig.model_parallel_enabled and pconfig.dp_shard_size <= 1:
        model.to(device)
        model._layout_fused_weights()
    model.train()
    engine = ParallelEngine(model, tokenizer, pconfig, cfg, device, mp_plan=mp_plan)
    if graph_step:
        engine.enable_graph_capture(warmup_steps=2)
    resume = None
    if cfg.config.resume_from:
        logger.info(f"Resuming from checkpoint {cfg.config.resume_from}")
        resume = engine.load_checkpoint(cfg.config.resume_from)
    B, T = cfg.model.per_device_batch_size, cfg.model.max_seq_length
    if synthetic:
        V = model.config.vocab_size
        train_loader = synthetic_data_loader(B, T, V, device=device, seed=seed, pconfig=pconfig,
                                             resume_state_dict=(resume or {}).get("dataloader_state"))
        eval_loader = synthetic_data_loader(B, T, V, device=device, seed=seed + 1, pconfig=pconfig,
                                            resume_state_dict=(resume or {}).get("eval_dataloader_state"))
        token_bytes = torch.ones(V, dtype=torch.int64)
    else:
        train_loader = dist_data_loader(tokenizer, B, T, split="train", device=device, pconfig=pconfig,
                                        resume_state_dict=(resume or {}).get("dataloader_state"))
        eval_loader = dist_data_loader(tokenizer, B, T, split="val", device=device, pconfig=pconfig,
                                       resume_state_dict=(resume or {}).get("eval_dataloader_state"))
    tokens_per_step = B * pconfig.data_world_size * T
    accum = cfg.config.grad_accum_steps
    start = (resume or {}).get("step", 0) + 1
    eval_state = (resume or {}).get("eval_dataloader_state")
    prof = scheduled_torch_profiler(enabled=cfg.engine.get("torch_profiler", False),
                                    trace_dir=cfg.engine.get("torch_profiler_trace_dir", "/tmp/parallel-traces"),
                                    rank=pconfig.rank, warmup_steps=cfg.engine.get("torch_profiler_warmup_steps", 1),
                                    active_steps=cfg.engine.get("torch_profiler_active_steps", 1))
    if prof is not None:
        prof.__enter__()
    cuda = device.type == "cuda"
    for step in range(start, cfg.config.max_steps + 1):
        t0 = time.time()
        ev0 = ev1 = None
        if cuda:
            ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            ev0.record()
        engine.reset_step_memory_stats()
        total = torch.tensor(0.0, device=device)
        dl_state = None
        if graph_step:
            # the micro-batches of the step stacked [accum, B, T]: one captured
            # step accumulates them and runs the optimizer
            batches = [next(train_loader) for _ in range(accum)]
            dl_state = batches[-1][2]
            if accum == 1:
                x, y = batches[0][0], batches[0][1]
            else:
                x, y = torch.stack([b[0] for b in batches]), torch.stack([b[1] for b in batches])
            total += engine.train_step(x, y)
        else:
            for _ in range(accum):
                x, y, dl_state = next(train_loader)
                loss = engine.forward(x, y).loss / accum
                engine.backward(loss)
                total += loss.detach()
            engine.step()
        if cuda:
            ev1.record()
        if prof is not None:
            prof.step()
        loss_log = engine.reduce_loss(total)
        mem = engine.step_memory_stats()
        coll_lines = engine.finish_step_collective_profile()
        dt = time.time() - t0
        tps = tokens_per_step * accum / dt
        dev_tps = None
        if cuda:
            ev1.synchronize()
            ms = torch.tensor([ev0.elapsed_time(ev1)], device=device, dtype=torch.float64)
            if dist.is_initialized():
                dist.all_reduce(ms, op=dist.ReduceOp.MAX)
            dev_tps = tokens_per_step * accum / (ms.item() / 1e3)
        gib = 1024 ** 3
        if pconfig.is_main_process:
            msg = (f"step {step:6d} | loss {loss_log.item():.4f} | lr {engine.lr:.2e} | tok/s {tps:,.0f} "
                   f"| fwd peak {mem['forward_peak_allocated_bytes'] / gib:.2f} GiB "
                   f"| bwd peak {mem['backward_peak_allocated_bytes'] / gib:.2f} GiB")
            if dev_tps is not None:
                msg += f" | device tok/s {dev_tps:,.0f}"
            logger.info(msg)
            for line in coll_lines:
                logger.info(line)
        wandb.log({"train/loss": loss_log.item(), "opt/lr": engine.lr, "speed/eff_tokens_per_sec": tps,
                   "memory/forward_peak_allocated_gib": mem["forward_peak_allocated_bytes"] / gib,
                   "memory/backward_peak_allocated_gib": mem["backward_peak_allocated_bytes"] / gib, "step": step},
                  step=step)
        if step % cfg.config.eval_interval == 0 or step == cfg.config.max_steps:
            logger.info("Evaling...")
            engine.sync_buffers()
            bpb, eval_state = eval_bpb(model, eval_loader, cfg.config.eval_steps, device, pconfig, engine.use_amp,
                                       engine.amp_dtype, token_bytes, loss_fn=engine.token_loss)
            if pconfig.is_main_process:
                logger.info(f"step {step:6d} | eval bpb {bpb:.4f}")
            wandb.log({"eval/loss": bpb, "step": step}, step=step)
        ci = cfg.config.checkpoint_interval
        if ci > 0 and step % ci == 0:
            path = Path(cfg.config.checkpoint_dir) / f"step-{step:08d}"
            logger.info(f"Saving checkpoint to {path}")
            engine.save_checkpoint(path, step=step, dataloader_state=dl_state, eval_dataloader_state=eval_state)
    if prof is not None:
        prof.__exit__(None, None, None)
    engine.release_graph()
    wandb.finish()
    dist_cleanup()


if __name__ == "__main__":
    main()
