"""Failure detection without any GPU fault: host-side failures among gloo ranks,
non-finite gradients, and fail-closed checkpoint validation."""
import os
import time
from datetime import timedelta

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp


def _peer_dies(rank, world, init_file, result_file):
    dist.init_process_group("gloo", init_method=f"file://{init_file}", rank=rank, world_size=world,
                            timeout=timedelta(seconds=3))
    t = torch.ones(4)
    dist.all_reduce(t)  # everyone healthy once
    if rank == 1:
        os._exit(0)  # leaves between steps, nothing in flight
    t0 = time.time()
    try:
        dist.all_reduce(t)
        outcome = "no-error"
    except Exception as exc:  # gloo surfaces a connection / timeout error
        outcome = f"error:{type(exc).__name__}"
    with open(result_file, "w") as f:
        f.write(f"{outcome}|{time.time() - t0:.1f}")


def test_survivor_gets_error_when_peer_leaves(tmp_path):
    init_file = str(tmp_path / "init")
    result = str(tmp_path / "res")
    ctx = mp.get_context("spawn")
    procs = [ctx.Process(target=_peer_dies, args=(r, 2, init_file, result)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=60)
        if p.is_alive():
            p.kill()
    outcome, secs = open(result).read().split("|")
    assert outcome.startswith("error:"), outcome
    assert float(secs) < 30


def test_nonfinite_gradients_raise_and_leave_params_untouched():
    from dist_utils import cpu_cfg
    from parallel_b200.models.config import resolve_config
    from parallel_b200.models.qwen3 import build_model
    from parallel_b200.parallel.engine import ParallelEngine
    from parallel_b200.state import ParallelConfig

    cfg = cpu_cfg()
    pc = ParallelConfig(cfg)
    pc.set_device_mesh("cpu")
    m = build_model(resolve_config("tiny-qwen3"), dtype=torch.float32, seed=0)
    eng = ParallelEngine(m, None, pc, cfg, torch.device("cpu"))
    tok = torch.randint(0, 1024, (2, 17))
    loss = eng.forward(tok[:, :-1], tok[:, 1:]).loss
    eng.backward(loss)
    next(m.parameters()).grad.view(-1)[0] = float("nan")
    before = {k: v.clone() for k, v in m.state_dict().items()}
    with pytest.raises(FloatingPointError):
        eng.step()
    for k, v in m.state_dict().items():
        torch.testing.assert_close(v, before[k], rtol=0, atol=0)
    assert all(p.grad is None for p in m.parameters())
