"""Against the reference implementation itself (CPU, gloo, 2 ranks, fp32): the
same training run gives the same losses, and exact-topology checkpoints load
across the two implementations and continue training identically.

Runs only where the unmodified reference is installed in ``baseline/_ref``
(its offline install for the benchmark's reference arm); skipped otherwise.
"""
import os

import pytest
import torch

from dist_utils import cpu_cfg, run_ranks

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
REF = os.path.join(ROOT, "baseline", "_ref")

pytestmark = pytest.mark.skipif(not os.path.isdir(os.path.join(REF, "parallel", "parallel")),
                                reason="reference not installed in baseline/_ref")

STEPS = 3


def _cfg(path, world, dp="dp_shard"):
    cfg = cpu_cfg(**{f"parallel.{dp}": world, "model.name": path, "engine.activation_checkpoint": "false",
                     "model.learning_rate": 1e-3})
    return cfg


def _ref_engine(path, world, dp="dp_shard"):
    import sys

    sys.path.insert(0, REF)
    sys.path.insert(0, ROOT)
    import bench

    bench._install_omegaconf_stub()
    from parallel.parallel.engine.engine import ParallelEngine as RefEngine
    from parallel.parallel.engine.model_loading import load_causal_lm as ref_load
    from parallel.parallel.state import ParallelConfig as RefPConfig

    cfg = _cfg(path, world, dp)
    for key in ("collectives", "optimizer_state_dtype", "sync_finite_check"):
        cfg.engine.pop(key, None)
    cfg.data.pop("synthetic", None)
    pc = RefPConfig(cfg)
    pc.set_device_mesh("cpu")
    pc.model_init_rngs(seed=42)
    model, plan = ref_load(cfg, pc)
    model.float()
    model.train()
    return RefEngine(model, None, pc, cfg, torch.device("cpu"), mp_plan=plan)


def _our_engine(path, world, dp="dp_shard"):
    from parallel_b200.models.loading import load_causal_lm
    from parallel_b200.parallel.engine import ParallelEngine
    from parallel_b200.state import ParallelConfig

    cfg = _cfg(path, world, dp)
    pc = ParallelConfig(cfg)
    pc.set_device_mesh("cpu")
    pc.model_init_rngs(seed=42)
    model, plan = load_causal_lm(cfg, pc, dtype=torch.float32)
    model.train()
    return ParallelEngine(model, None, pc, cfg, torch.device("cpu"), mp_plan=plan)


def _train(engine, data, rank, world, steps):
    losses = []
    for tok in data[:steps]:
        B = tok.shape[0] // world
        mine = tok[rank * B:(rank + 1) * B]
        loss = engine.forward(mine[:, :-1], mine[:, 1:]).loss
        engine.backward(loss)
        engine.step()
        losses.append(float(engine.reduce_loss(loss.detach())))
    return losses


def _worker(rank, world, tmp, out, name="tiny-qwen3", dp="dp_shard"):
    import torch.distributed as dist

    from parallel_b200.models.config import resolve_config
    from parallel_b200.models.loading import save_pretrained
    from parallel_b200.models.qwen3 import build_model

    path = os.path.join(tmp, "init")
    if rank == 0:
        save_pretrained(build_model(resolve_config(name), dtype=torch.float32, seed=0), path)
    dist.barrier()
    g = torch.Generator().manual_seed(3)
    data = [torch.randint(0, 1024, (2 * world, 65), generator=g) for _ in range(STEPS + 1)]

    ours = _our_engine(path, world, dp)
    ref = _ref_engine(path, world, dp)
    l_ours = _train(ours, data, rank, world, STEPS)
    l_ref = _train(ref, data, rank, world, STEPS)

    # exact-topology checkpoints, each loaded by the other implementation
    ours.save_checkpoint(os.path.join(tmp, "ours"), step=STEPS)
    ref.save_checkpoint(os.path.join(tmp, "ref"), step=STEPS)
    ours_b = _our_engine(path, world, dp)
    ours_b.load_checkpoint(os.path.join(tmp, "ref"))
    ref_b = _ref_engine(path, world, dp)
    ref_b.load_checkpoint(os.path.join(tmp, "ours"))
    # portable full-model files, each loaded by the other implementation: the
    # loaded weights equal the writer's weights exactly
    ours.save_full_model(os.path.join(tmp, "ours_full.pt"))
    ref.save_full_model(os.path.join(tmp, "ref_full.pt"))
    dist.barrier()
    ours_c = _our_engine(path, world, dp)
    ours_c.load_full_model(os.path.join(tmp, "ref_full.pt"))
    ref_c = _ref_engine(path, world, dp)
    ref_c.load_full_model(os.path.join(tmp, "ours_full.pt"))
    # state_dict() is collective; the full dicts land on rank 0
    pairs = [(ours_c.state_dict(), ref.state_dict()), (ref_c.state_dict(), ours.state_dict())]
    worst, same_keys = 0.0, True
    if rank == 0:
        for got, src in pairs:
            same_keys = same_keys and sorted(got) == sorted(src)
            worst = max([worst] + [(got[k].float() - v.float()).abs().max().item() for k, v in src.items() if k in got])
    nxt = data[STEPS:]
    cont = {"ours": _train(ours, nxt, rank, world, 1), "ref": _train(ref, nxt, rank, world, 1),
            "ours_from_ref": _train(ours_b, nxt, rank, world, 1), "ref_from_ours": _train(ref_b, nxt, rank, world, 1)}
    if rank == 0:
        torch.save({"ours": l_ours, "ref": l_ref, "cont": cont, "full_worst": worst, "full_keys": same_keys}, out)
    dist.barrier()


@pytest.mark.parametrize("name,dp", [("tiny-qwen3", "dp_shard"), ("tiny-qwen3-moe", "dp_shard"),
                                     ("tiny-qwen3", "dp_replicate")])
def test_losses_and_checkpoints_interchange_with_the_reference(tmp_path, name, dp):
    out = str(tmp_path / "res.pt")
    run_ranks(_worker, 2, str(tmp_path), out, name, dp)
    res = torch.load(out, weights_only=False)
    # portable full-model files: same keys, and after loading the other
    # implementation's file both hold the same trained weights
    assert res["full_keys"] and res["full_worst"] == 0.0, res
    # fp32 on CPU: the same losses step by step (bit-identical on this image)
    for a, b in zip(res["ours"], res["ref"]):
        assert abs(a - b) < 1e-5 * max(1.0, abs(b)), res
    c = res["cont"]
    # a step after loading the other implementation's checkpoint equals the step
    # that implementation takes itself
    assert abs(c["ours_from_ref"][0] - c["ref"][0]) < 1e-5, c
    assert abs(c["ref_from_ours"][0] - c["ours"][0]) < 1e-5, c
