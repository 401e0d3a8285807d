"""FSDP over gloo ranks equals unsharded single-process training (fp32)."""
import copy

import pytest
import torch

from dist_utils import cpu_cfg, run_ranks

STEPS = 10


def _tokens(world, B=2, S=128, V=1024, seed=0):
    g = torch.Generator().manual_seed(seed)
    return [torch.randint(0, V, (world * B, S + 1), generator=g) for _ in range(STEPS)]


def _single_process_losses(data, accum=1, clip=1.0):
    from parallel_b200.models.config import resolve_config
    from parallel_b200.models.qwen3 import build_model
    from parallel_b200.parallel.optim import FusedAdamW

    m = build_model(resolve_config("tiny-qwen3"), dtype=torch.float32, seed=0)
    opt = FusedAdamW(list(m.parameters()), lr=1e-3, betas=(0.9, 0.999), weight_decay=0.01)
    losses = []
    for tok in data:
        total = 0.0
        micro = tok.chunk(accum, 0)
        for mb in micro:
            loss = m(mb[:, :-1], labels=mb[:, 1:]).loss / accum
            loss.backward()
            total += loss.item()
        if clip > 0:
            torch.nn.utils.clip_grad_norm_(list(m.parameters()), clip)
        opt.step()
        opt.zero_grad(set_to_none=True)
        losses.append(total)
    return losses, m


def _fsdp_worker(rank, world, data, ckpt, overlap, accum, out_q):
    from parallel_b200.models.config import resolve_config
    from parallel_b200.models.qwen3 import build_model
    from parallel_b200.parallel.engine import ParallelEngine
    from parallel_b200.state import ParallelConfig

    cfg = cpu_cfg(**{"parallel.dp_shard": world, "engine.activation_checkpoint": str(ckpt).lower(),
                     "engine.overlap_backward_reductions": str(overlap).lower(), "config.grad_accum_steps": accum})
    pc = ParallelConfig(cfg)
    pc.set_device_mesh("cpu")
    m = build_model(resolve_config("tiny-qwen3"), dtype=torch.float32, seed=0)
    eng = ParallelEngine(m, None, pc, cfg, torch.device("cpu"))
    losses = []
    for tok in data:
        B = tok.shape[0] // world
        mine = tok[rank * B:(rank + 1) * B]
        total = torch.zeros(())
        for mb in mine.chunk(accum, 0):
            loss = eng.forward(mb[:, :-1], mb[:, 1:]).loss / accum
            eng.backward(loss)
            total += loss.detach()
        eng.step()
        losses.append(eng.reduce_loss(total).item())
    full = eng.state_dict()
    if rank == 0:
        torch.save({"losses": losses, "state": full}, out_q)


@pytest.mark.parametrize("ckpt,overlap,accum", [(True, True, 1), (False, True, 2), (True, False, 1)])
def test_fsdp_matches_single_process(tmp_path, ckpt, overlap, accum):
    """tiny Qwen3, dp_shard=2, fp32, 10 AdamW steps; loss equal to 1e-5."""
    world = 2
    data = _tokens(world)
    out = str(tmp_path / "out.pt")
    run_ranks(_fsdp_worker, world, data, ckpt, overlap, accum, out)
    got = torch.load(out, weights_only=False)
    ref_losses, ref_model = _single_process_losses([t for t in data], accum=accum)
    for a, b in zip(got["losses"], ref_losses):
        assert abs(a - b) < 1e-5, (got["losses"], ref_losses)
    ref_sd = ref_model.state_dict()
    for k, v in got["state"].items():
        torch.testing.assert_close(v, ref_sd[k], rtol=1e-3, atol=2e-4)


def _layout_worker(rank, world, out):
    from parallel_b200.models.config import resolve_config
    from parallel_b200.models.qwen3 import build_model
    from parallel_b200.parallel.engine import ParallelEngine
    from parallel_b200.state import ParallelConfig

    cfg = cpu_cfg(**{"parallel.dp_shard": world})
    pc = ParallelConfig(cfg)
    pc.set_device_mesh("cpu")
    m = build_model(resolve_config("tiny-qwen3"), dtype=torch.float32, seed=0)
    eng = ParallelEngine(m, None, pc, cfg, torch.device("cpu"))
    f = eng.fsdp_wrapper
    assert f.is_active and len(f.units) == 3  # root + 2 layers
    root = f.units[0]
    assert root.module is m and not root.reshard_after_forward
    names = [meta.name for meta in root.param_metas]
    assert names == ["model.embed_tokens.weight", "model.norm.weight"]  # tied lm_head shares the embedding
    lay = f.checkpoint_layout()
    p0 = lay["units"][1]["parameters"][0]
    assert p0["names"] == ["model.layers.0.self_attn.q_proj.weight"]
    assert p0["placements"] == ["S(0)"] and p0["local_shape"] == [128, 256]
    if rank == 0:
        torch.save(lay, out)


def test_fsdp_units_and_layout(tmp_path):
    out = str(tmp_path / "lay.pt")
    run_ranks(_layout_worker, 2, out)
    lay = torch.load(out, weights_only=False)
    assert lay["state_dict_keys"][0] == "model.embed_tokens.weight"


def _replicate_worker(rank, world, data, out_q):
    from parallel_b200.models.config import resolve_config
    from parallel_b200.models.qwen3 import build_model
    from parallel_b200.parallel.engine import ParallelEngine
    from parallel_b200.state import ParallelConfig

    cfg = cpu_cfg(**{"parallel.dp_replicate": world})
    pc = ParallelConfig(cfg)
    pc.set_device_mesh("cpu")
    m = build_model(resolve_config("tiny-qwen3"), dtype=torch.float32, seed=0)
    eng = ParallelEngine(m, None, pc, cfg, torch.device("cpu"))
    losses = []
    for tok in data:
        B = tok.shape[0] // world
        mine = tok[rank * B:(rank + 1) * B]
        loss = eng.forward(mine[:, :-1], mine[:, 1:]).loss
        eng.backward(loss)
        eng.step()
        losses.append(eng.reduce_loss(loss.detach()).item())
    if rank == 0:
        torch.save({"losses": losses, "state": {k: v.detach().clone() for k, v in m.state_dict().items()}}, out_q)


def test_dp_replicate_matches_single_process(tmp_path):
    """Replicated data parallelism (gradient all-reduce mean, one participation
    bitmap per step) equals single-process training on the global batch."""
    world = 2
    data = _tokens(world)[:4]
    out = str(tmp_path / "rep.pt")
    run_ranks(_replicate_worker, world, data, out)
    got = torch.load(out, weights_only=False)
    ref_losses, ref_model = _single_process_losses(data)
    for a, b in zip(got["losses"], ref_losses):
        assert abs(a - b) < 1e-5, (got["losses"], ref_losses)
    ref_sd = ref_model.state_dict()
    for k, v in got["state"].items():
        torch.testing.assert_close(v, ref_sd[k], rtol=1e-3, atol=2e-4)
