"""TP / SP / EP (and their FSDP composition) against single-process training (CPU, gloo, fp32).

Mirrors the reference's HF-parity tests: loss equal, per-shard gradients,
router gradients identical across TP ranks, global grad norm, portable
state equal after optimizer steps, checkpoint round trips.
"""
import os

import pytest
import torch

from dist_utils import cpu_cfg, run_ranks

B, S = 2, 32


def _save_ref_model(path, name):
    from parallel_b200.models.config import resolve_config
    from parallel_b200.models.loading import save_pretrained
    from parallel_b200.models.qwen3 import build_model

    cfg = resolve_config(name)
    m = build_model(cfg, dtype=torch.float32, seed=0)
    save_pretrained(m, path)
    return m


def _data(V=1024, steps=3, world=1):
    g = torch.Generator().manual_seed(123)
    return [torch.randint(0, V, (B * world, S + 1), generator=g) for _ in range(steps)]


def _reference(path, name, data, dp=1):
    """Single-process fp32 training with the model-parallel loss convention
    (unshifted labels, router aux loss added)."""
    from parallel_b200.models.loading import read_state_dict
    from parallel_b200.models.config import ModelConfig
    from parallel_b200.models.qwen3 import build_model
    from parallel_b200.ops.moe import load_balancing_loss
    from parallel_b200.parallel.optim import FusedAdamW

    cfg = ModelConfig.from_pretrained(path)
    m = build_model(cfg, dtype=torch.float32, seed=0)
    m.load_state_dict(read_state_dict(path))
    m._layout_fused_weights()
    opt = FusedAdamW(list(m.parameters()), lr=1e-3, betas=(0.9, 0.999), weight_decay=0.01)
    losses, grads, norms = [], [], []
    for tok in data:
        # data-parallel ranks each see their own micro-batch (and their own
        # router statistics); gradients and the logged loss are averaged
        total = 0.0
        for chunk in tok.chunk(dp, 0):
            x, y = chunk[:, :-1], chunk[:, 1:]
            loss = m(x, labels=y, shift_labels=False).loss / dp
            loss.backward()
            total += loss.item()
        grads.append({n: p.grad.clone() for n, p in m.named_parameters()})
        norms.append(torch.nn.utils.clip_grad_norm_(list(m.parameters()), 1.0).item())
        opt.step()
        opt.zero_grad(set_to_none=True)
        losses.append(total)
    return losses, grads, norms, {k: v.clone() for k, v in m.state_dict().items()}


def _mp_worker(rank, world, path, data, par, out, extra=None):
    from parallel_b200.models.loading import load_causal_lm
    from parallel_b200.parallel.engine import ParallelEngine
    from parallel_b200.state import ParallelConfig

    over = {"model.name": path, "model.output_router_logits": "true"}
    over.update({f"parallel.{k}": v for k, v in par.items()})
    over.update(extra or {})
    cfg = cpu_cfg(**over)
    pc = ParallelConfig(cfg)
    pc.set_device_mesh("cpu")
    model, plan = load_causal_lm(cfg, pc, dtype=torch.float32)
    eng = ParallelEngine(model, None, pc, cfg, torch.device("cpu"), mp_plan=plan)
    dp = pc.data_world_size
    drank = pc.data_rank
    losses, local_grads, norms = [], [], []
    for tok in data:
        b = tok.shape[0] // dp
        mine = tok[drank * b:(drank + 1) * b]
        loss = eng.forward(mine[:, :-1], mine[:, 1:]).loss
        eng.backward(loss)
        if not eng.fsdp_wrapper.is_active and dp == 1:
            # (with data-parallel replicas the grads are averaged in step(), not here)
            local_grads.append({n: p.grad.clone() for n, p in model.named_parameters() if p.grad is not None})
        eng.step()
        norms.append(float(eng.last_grad_norm))
        losses.append(eng.reduce_loss(loss).item())
    full = eng.state_dict()
    # exact-topology checkpoint round trip into a fresh engine
    ck = os.path.join(os.path.dirname(out), "ckpt")
    eng.save_checkpoint(ck, step=len(data))
    model2, plan2 = load_causal_lm(cfg, pc, dtype=torch.float32)
    eng2 = ParallelEngine(model2, None, pc, cfg, torch.device("cpu"), mp_plan=plan2)
    info = eng2.load_checkpoint(ck)
    full2 = eng2.state_dict()
    # both continue with one more step on the same batch: the resumed engine
    # (weights, optimizer moments and step count) takes the original's step
    cont = []
    for e in (eng, eng2):
        mine = data[0][drank * b:(drank + 1) * b]
        loss = e.forward(mine[:, :-1], mine[:, 1:]).loss
        e.backward(loss)
        e.step()
        cont.append(e.reduce_loss(loss).item())
    after = [eng.state_dict(), eng2.state_dict()]
    torch.save({"rank": rank, "losses": losses, "grads": local_grads, "norms": norms, "tp_rank":
                pc._mesh_rank("tp"), "plan": plan.checkpoint_metadata(), "full": full, "full2": full2,
                "step": info["step"], "cont": cont, "after": after}, out.replace(".pt", f"-{rank}.pt"))


def _check(tmp_path, name, par, world, extra=None):
    path = str(tmp_path / "model")
    _save_ref_model(path, name)
    dp = par.get("dp_shard", 1) * par.get("dp_replicate", 1)
    data = _data(world=dp)
    out = str(tmp_path / "res.pt")
    run_ranks(_mp_worker, world, path, data, par, out, extra)
    ref_losses, ref_grads, ref_norms, ref_state = _reference(path, name, data, dp)
    res = [torch.load(out.replace(".pt", f"-{r}.pt"), weights_only=False) for r in range(world)]
    for r in res:
        torch.testing.assert_close(torch.tensor(r["losses"]), torch.tensor(ref_losses), rtol=1e-5, atol=1e-5)
        torch.testing.assert_close(torch.tensor(r["norms"]), torch.tensor(ref_norms), rtol=2e-5, atol=1e-6)
        assert r["step"] == len(data)
    root = res[0]
    for k, v in root["full"].items():
        torch.testing.assert_close(v, ref_state[k], rtol=1e-3, atol=2e-4)
        torch.testing.assert_close(root["full2"][k], v, rtol=0, atol=0)
    # the resumed engine continues exactly like the original
    assert root["cont"][0] == root["cont"][1], root["cont"]
    for k, v in root["after"][0].items():
        torch.testing.assert_close(root["after"][1][k], v, rtol=0, atol=0)
    # per-shard gradients (model-parallel without FSDP)
    if root["grads"]:
        from parallel_b200.parallel.model_parallel.plan import ParameterPlacement  # noqa: F401

        placements = {p["pattern"]: p for p in root["plan"]["parameters"]}
        import fnmatch

        tp = par["tp"]
        for r in res:
            for step, g in enumerate(r["grads"]):
                for n, loc in g.items():
                    pat = next(p for p in placements.values() if fnmatch.fnmatchcase(n, p["pattern"]))
                    full = ref_grads[step][n]
                    if pat["shard_dim"] is not None:
                        full = full.chunk(tp, dim=pat["shard_dim"])[r["tp_rank"]]
                    torch.testing.assert_close(loc, full, rtol=2e-2, atol=1e-4)
        # router gradients bit-identical across TP ranks
        for n in res[0]["grads"][0]:
            if n.endswith("mlp.gate.weight"):
                torch.testing.assert_close(res[0]["grads"][0][n], res[1]["grads"][0][n], rtol=0, atol=0)


@pytest.mark.parametrize("sp", [1, 2])
def test_dense_tp(tmp_path, sp):
    _check(tmp_path, "tiny-qwen3", {"tp": 2, "sp": sp}, 2)


@pytest.mark.parametrize("sp", [1, 2])
def test_moe_tp_ep(tmp_path, sp):
    _check(tmp_path, "tiny-qwen3-moe", {"tp": 2, "ep": 2, "sp": sp}, 2)


@pytest.mark.parametrize("sp", [1, 2])
def test_moe_tp_ep_fsdp_composition(tmp_path, sp):
    _check(tmp_path, "tiny-qwen3-moe", {"tp": 2, "ep": 2, "sp": sp, "dp_shard": 2}, 4)


@pytest.mark.parametrize("sp", [1, 2])
def test_dense_tp_fsdp_composition(tmp_path, sp):
    """The dense benchmark layout (Qwen3-8B: tp = sp over FSDP) at tp=2 x dp_shard=2."""
    _check(tmp_path, "tiny-qwen3", {"tp": 2, "sp": sp, "dp_shard": 2}, 4)


def test_dense_tp_sp_fsdp_cpu_offload(tmp_path):
    """FSDP shards in host memory under TP+SP (engine.cpu_offload)."""
    _check(tmp_path, "tiny-qwen3", {"tp": 2, "sp": 2, "dp_shard": 2}, 4, {"engine.cpu_offload": "true"})


def test_dense_tp_sp_with_dp_replicate(tmp_path):
    """TP+SP with replicated data parallelism (gradient all-reduce over the
    replicas, no FSDP) at tp=2 x dp_replicate=2."""
    _check(tmp_path, "tiny-qwen3", {"tp": 2, "sp": 2, "dp_replicate": 2}, 4)


@pytest.mark.parametrize("overlap", ["true", "false"])
def test_moe_tp_ep_sp_fsdp_composition_with_activation_checkpointing(tmp_path, overlap):
    """The recomputed layer forward in the backward routes the layer's TP-summed
    parameters (norms, q/k-norm, router) through the packed reduction too; with
    the FSDP reductions overlapped with the backward or deferred to its end."""
    _check(tmp_path, "tiny-qwen3-moe", {"tp": 2, "ep": 2, "sp": 2, "dp_shard": 2}, 4,
           {"engine.activation_checkpoint": "true", "engine.overlap_backward_reductions": overlap})


def test_plan_validation():
    from parallel_b200.models.config import resolve_config
    from parallel_b200.parallel.model_parallel import build_model_parallel_plan, supported_model_types

    class PC:
        tp_size, sp_size, ep_size, expert_tp_size, dp_shard_size = 3, 1, 1, 1, 1

    assert supported_model_types() == ("qwen3", "qwen3_moe")
    with pytest.raises(ValueError, match="divisible"):
        build_model_parallel_plan(resolve_config("tiny-qwen3"), PC())

    class PC2(PC):
        tp_size, ep_size = 2, 1

    with pytest.raises(ValueError, match="tp > 1 and ep > 1"):
        build_model_parallel_plan(resolve_config("tiny-qwen3-moe"), PC2())


def test_route_localization():
    from parallel_b200.parallel.model_parallel import ExpertPartition

    p = ExpertPartition(num_experts=8, ep_size=2, ep_rank=1)
    idx = torch.tensor([[0, 5], [7, 3]])
    sc = torch.tensor([[0.5, 0.25], [0.125, 1.0]])
    li, ls, mask = p.localize_routes(idx, sc)
    assert li.tolist() == [[4, 1], [3, 4]]
    assert ls.tolist() == [[0.0, 0.25], [0.125, 0.0]]
    assert mask.tolist() == [[False, True], [True, False]]


@pytest.mark.parametrize("name,tp,sp,ep", [("Qwen/Qwen3-8B", 4, 4, 1), ("Qwen/Qwen3-30B-A3B", 4, 4, 4),
                                         ("Qwen/Qwen3-0.6B", 2, 2, 1)])
def test_benchmark_configurations_have_valid_plans(name, tp, sp, ep):
    """The model-parallel configurations of the benchmarks (8B tp=sp=4, 30B-A3B
    tp=sp=ep=4) build plans that cover every parameter of the local-shape model
    with the expected shard shapes."""
    from parallel_b200.models.config import resolve_config
    from parallel_b200.models.qwen3 import Qwen3ForCausalLM
    from parallel_b200.parallel.model_parallel import build_model_parallel_plan

    cfg = resolve_config(name, num_hidden_layers=1)

    class PC:
        tp_size, sp_size, ep_size, expert_tp_size, dp_shard_size = tp, sp, ep, 1, 2

    plan = build_model_parallel_plan(cfg, PC())
    with torch.device("meta"):
        local = Qwen3ForCausalLM(cfg, tp=tp, ep=ep)
    params = dict(local.named_parameters())
    plan.validate_parameter_coverage(params)
    q = params["model.layers.0.self_attn.q_proj.weight"]
    assert q.shape == (cfg.num_attention_heads * cfg.head_dim // tp, cfg.hidden_size)
    if ep > 1:
        gu = params["model.layers.0.mlp.experts.gate_up_proj"]
        assert gu.shape[0] == cfg.num_experts // ep


def _pack_worker(rank, world, path, sp, out):
    import torch.distributed as dist

    from parallel_b200.models.loading import load_causal_lm
    from parallel_b200.parallel.engine import ParallelEngine
    from parallel_b200.state import ParallelConfig

    cfg = cpu_cfg(**{"model.name": path, "parallel.tp": 2, "parallel.sp": sp})
    pc = ParallelConfig(cfg)
    pc.set_device_mesh("cpu")
    model, plan = load_causal_lm(cfg, pc, dtype=torch.float32)
    eng = ParallelEngine(model, None, pc, cfg, torch.device("cpu"), mp_plan=plan)
    packs = [l._tp_grad_pack for l in model.model.layers]
    calls = []
    real = dist.all_reduce

    def counting(t, *a, **k):
        calls.append(t.numel())
        return real(t, *a, **k)

    tok = _data(steps=1)[0]
    loss = eng.forward(tok[:, :-1], tok[:, 1:]).loss
    dist.all_reduce = counting
    try:
        eng.backward(loss)
    finally:
        dist.all_reduce = real
    grads = {n: p.grad.clone() for n, p in model.named_parameters()
             if p.grad is not None and plan.placement_for_parameter(n).shard_dim is None}
    torch.save({"numels": [p.numel for p in packs], "names": [p.rel_names for p in packs], "calls": calls,
                "hooks": len(eng.mp_wrapper._tp_gradient_hook_handles), "grads": grads},
               out.replace(".pt", f"-{rank}.pt"))


@pytest.mark.parametrize("sp", [1, 2])
def test_sum_tp_gradients_are_reduced_once_per_layer(tmp_path, sp):
    """Each decoder layer's TP-summed parameters (q/k-norm; + both layer norms
    under SP) are reduced in one packed all-reduce in the backward instead of
    one per parameter; only the final norm (SP) keeps a per-parameter hook.
    The reduced gradients are identical on both TP ranks (their correctness
    against single-process training is the parity tests' job)."""
    path = str(tmp_path / "model")
    cfg = _save_ref_model(path, "tiny-qwen3").config
    out = str(tmp_path / "res.pt")
    run_ranks(_pack_worker, 2, path, sp, out)
    res = [torch.load(out.replace(".pt", f"-{r}.pt"), weights_only=False) for r in range(2)]
    H, D, L = cfg.hidden_size, cfg.head_dim, cfg.num_hidden_layers
    want = 2 * D + (2 * H if sp > 1 else 0)
    r0 = res[0]
    assert r0["numels"] == [want] * L
    expect = {"self_attn.q_norm.weight", "self_attn.k_norm.weight"}
    if sp > 1:
        expect |= {"input_layernorm.weight", "post_attention_layernorm.weight"}
    assert all(set(n) == expect for n in r0["names"])
    assert r0["calls"].count(want) == L
    assert r0["hooks"] == (1 if sp > 1 else 0)
    for n, g in r0["grads"].items():
        torch.testing.assert_close(res[1]["grads"][n], g, rtol=0, atol=0)
