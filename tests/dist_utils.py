"""Helpers for multi-process CPU tests on gloo (file:// rendezvous)."""
from __future__ import annotations

import os
import tempfile
import traceback

import torch
import torch.distributed as dist
import torch.multiprocessing as mp


def _entry(rank, world, init_file, fn, args, err_dir):
    os.environ["RANK"] = str(rank)
    os.environ["WORLD_SIZE"] = str(world)
    os.environ["LOCAL_RANK"] = str(rank)
    torch.set_num_threads(1)
    try:
        dist.init_process_group("gloo", init_method=f"file://{init_file}", rank=rank, world_size=world)
        fn(rank, world, *args)
    except BaseException:
        with open(os.path.join(err_dir, f"rank{rank}.err"), "w") as f:
            f.write(traceback.format_exc())
        raise
    finally:
        if dist.is_initialized():
            dist.destroy_process_group()


def run_ranks(fn, world: int, *args) -> None:
    """Run ``fn(rank, world, *args)`` on ``world`` gloo ranks; re-raise failures."""
    with tempfile.TemporaryDirectory() as d:
        init_file = os.path.join(d, "init")
        try:
            mp.spawn(_entry, args=(world, init_file, fn, args, d), nprocs=world, join=True)
        except Exception as exc:
            msgs = []
            for r in range(world):
                p = os.path.join(d, f"rank{r}.err")
                if os.path.exists(p):
                    msgs.append(open(p).read())
            raise AssertionError("\n".join(msgs) or str(exc)) from exc


def cpu_cfg(**over):
    from parallel_b200.config import from_dotlist, load_cfg, merge

    base = ["config.device_type=cpu", "config.backend=gloo", "config.use_amp=false", "model.learning_rate=1e-3",
            "model.clip_grad_norm=1.0", "optim.weight_decay=0.01"]
    return merge(load_cfg(argv=[]), from_dotlist(base + [f"{k}={v}" for k, v in over.items()]))
