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


def _fsdp_worker(rank, world, data, ckpt, overlap, accum, out_q, offload=False, every_n=1):
    from parallel_b200.models.config import resolve_config
    from parallel_b200.models.qwen3 import build_model
    from parallel_b200.parallel.engine import ParallelEngine
    from parallel_b200.state import ParallelConfig

    cfg = cpu_cfg(**{"parallel.dp_shard": world, "engine.activation_checkpoint": str(ckpt).lower(),
                     "engine.overlap_backward_reductions": str(overlap).lower(), "config.grad_accum_steps": accum,
                     "engine.cpu_offload": str(offload).lower(), "engine.checkpoint_every_n": every_n})
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
    roots = {id(u) for u in eng.fsdp_wrapper.root_units}
    recompute = [u.use_activation_checkpoint for u in eng.fsdp_wrapper.units if id(u) not in roots]
    if rank == 0:
        torch.save({"losses": losses, "state": full, "recompute": recompute}, out_q)


def test_fsdp_checkpoint_every_n_layers(tmp_path):
    """engine.checkpoint_every_n=2: only every second layer unit recomputes its
    forward in the backward; training still equals single-process training."""
    world = 2
    data = _tokens(world)[:3]
    out = str(tmp_path / "every_n.pt")
    run_ranks(_fsdp_worker, world, data, True, True, 1, out, False, 2)
    got = torch.load(out, weights_only=False)
    n = len(got["recompute"])
    assert n >= 2 and got["recompute"] == [i % 2 == 0 for i in range(n)], got["recompute"]
    ref_losses, ref_model = _single_process_losses(data)
    for a, b in zip(got["losses"], ref_losses):
        assert abs(a - b) < 1e-5, (got["losses"], ref_losses)
    ref_sd = ref_model.state_dict()
    for k, v in got["state"].items():
        torch.testing.assert_close(v, ref_sd[k], rtol=1e-3, atol=2e-4)


@pytest.mark.parametrize("ckpt,overlap,accum,offload", [(True, True, 1, False), (False, True, 2, False),
                                                        (True, False, 1, False), (False, True, 2, True)])
def test_fsdp_matches_single_process(tmp_path, ckpt, overlap, accum, offload):
    """tiny Qwen3, dp_shard=2, fp32, 10 AdamW steps; loss equal to 1e-5
    (also with the shards and their gradients kept in host memory: cpu_offload)."""
    world = 2
    data = _tokens(world)
    out = str(tmp_path / "out.pt")
    run_ranks(_fsdp_worker, world, data, ckpt, overlap, accum, out, offload)
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


def _hybrid_worker(rank, world, data, out_q):
    from parallel_b200.models.config import resolve_config
    from parallel_b200.models.qwen3 import build_model
    from parallel_b200.parallel.engine import ParallelEngine
    from parallel_b200.state import ParallelConfig

    cfg = cpu_cfg(**{"parallel.dp_replicate": 2, "parallel.dp_shard": 2})
    pc = ParallelConfig(cfg)
    pc.set_device_mesh("cpu")
    m = build_model(resolve_config("tiny-qwen3"), dtype=torch.float32, seed=0)
    eng = ParallelEngine(m, None, pc, cfg, torch.device("cpu"))
    losses = []
    r = pc.data_rank
    for tok in data:
        B = tok.shape[0] // world
        mine = tok[r * B:(r + 1) * B]
        loss = eng.forward(mine[:, :-1], mine[:, 1:]).loss
        eng.backward(loss)
        eng.step()
        losses.append(eng.reduce_loss(loss.detach()).item())
    state = eng.state_dict()
    # exact-topology checkpoint (shard files written by replica 0 only), then
    # a fresh engine continues exactly like this one
    import os

    ck = os.path.join(os.path.dirname(out_q), "hsdp_ckpt")
    eng.save_checkpoint(ck, step=len(data))
    m2 = build_model(resolve_config("tiny-qwen3"), dtype=torch.float32, seed=1)
    eng2 = ParallelEngine(m2, None, pc, cfg, torch.device("cpu"))
    eng2.load_checkpoint(ck)
    nxt = data[0][r * (data[0].shape[0] // world):(r + 1) * (data[0].shape[0] // world)]
    cont = []
    for e in (eng, eng2):
        loss = e.forward(nxt[:, :-1], nxt[:, 1:]).loss
        e.backward(loss)
        e.step()
        cont.append(e.reduce_loss(loss.detach()).item())
    after = [eng.state_dict(), eng2.state_dict()]
    if rank == 0:
        files = sorted(f for f in os.listdir(ck) if f.startswith("model-"))
        torch.save({"losses": losses, "state": state, "cont": cont, "after": after, "files": files}, out_q)


def test_hybrid_replicate_over_fsdp_matches_single_process(tmp_path):
    """dp_replicate=2 x dp_shard=2: FSDP inside each replica, the reduced shard
    gradients averaged over the replicas, equals single-process training."""
    world = 4
    data = _tokens(world)[:3]
    out = str(tmp_path / "hsdp.pt")
    run_ranks(_hybrid_worker, world, data, out)
    got = torch.load(out, weights_only=False)
    ref_losses, ref_model = _single_process_losses(data)
    for a, b in zip(got["losses"], ref_losses):
        assert abs(a - b) < 1e-5, (got["losses"], ref_losses)
    ref_sd = ref_model.state_dict()
    for k, v in got["state"].items():
        torch.testing.assert_close(v, ref_sd[k], rtol=1e-3, atol=2e-4)
    assert got["files"] == ["model-shard-00000.pt", "model-shard-00001.pt"], got["files"]
    assert got["cont"][0] == got["cont"][1], got["cont"]
    for k, v in got["after"][0].items():
        torch.testing.assert_close(got["after"][1][k], v, rtol=0, atol=0)


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


class _ToyLayer(torch.nn.Module):
    def __init__(self):
        super().__init__()
        self.a = torch.nn.Linear(16, 16, bias=False)
        self.b = torch.nn.Linear(16, 16, bias=False)
        self.never = torch.nn.Linear(16, 16, bias=False)  # unused on every rank
        self.use_b = True

    def forward(self, x):
        y = x + self.a(x)
        return y + self.b(torch.tanh(y)) if self.use_b else y


class _Toy(torch.nn.Module):
    """Rank-divergent graph: layer 0's ``b`` runs only where ``use_b`` is set."""

    def __init__(self, seed=0):
        super().__init__()
        torch.manual_seed(seed)
        self.embed = torch.nn.Embedding(64, 16)
        self.layers = torch.nn.ModuleList([_ToyLayer(), _ToyLayer()])
        self.head = torch.nn.Linear(16, 64, bias=False)

    def forward(self, input_ids, labels=None):
        from types import SimpleNamespace

        x = self.embed(input_ids)
        for layer in self.layers:
            x = layer(x)
        logits = self.head(x)
        loss = torch.nn.functional.cross_entropy(logits.reshape(-1, 64), labels.reshape(-1))
        return SimpleNamespace(loss=loss, logits=logits)


def _unused_data(world, steps=3):
    g = torch.Generator().manual_seed(5)
    return [torch.randint(0, 64, (world * 2, 9), generator=g) for _ in range(steps)]


def _unused_worker(rank, world, data, out, ckpt="false"):
    from parallel_b200.parallel.engine import ParallelEngine
    from parallel_b200.state import ParallelConfig

    cfg = cpu_cfg(**{"parallel.dp_shard": world, "engine.find_unused_parameters": "true",
                     "engine.activation_checkpoint": ckpt, "model.learning_rate": 1e-2})
    pc = ParallelConfig(cfg)
    pc.set_device_mesh("cpu")
    m = _Toy()
    m.layers[0].use_b = rank == 0
    eng = ParallelEngine(m, None, pc, cfg, torch.device("cpu"))
    for tok in data:
        mine = tok[rank * 2:(rank + 1) * 2]
        loss = eng.forward(mine[:, :-1], mine[:, 1:]).loss
        eng.backward(loss)
        eng.step()
    full = eng.state_dict()
    if rank == 0:
        torch.save(full, out)


@pytest.mark.parametrize("ckpt", ["false", "true"])
def test_fsdp_rank_divergent_unused_parameters(tmp_path, ckpt):
    """find_unused_parameters (with and without activation checkpointing): a
    parameter used on some ranks gets the mean over all ranks (zeros where
    unused); one unused everywhere keeps grad=None and is left untouched by
    AdamW (no weight decay either)."""
    from parallel_b200.parallel.optim import FusedAdamW

    world = 2
    data = _unused_data(world)
    out = str(tmp_path / "unused.pt")
    run_ranks(_unused_worker, world, data, out, ckpt)
    got = torch.load(out, weights_only=False)
    ref = _Toy()
    init_never = ref.layers[1].never.weight.detach().clone()
    opt = FusedAdamW(list(ref.parameters()), lr=1e-2, betas=(0.9, 0.999), weight_decay=0.01)
    for tok in data:
        grads = []
        for r in range(world):
            ref.layers[0].use_b = r == 0
            ref.zero_grad(set_to_none=True)
            mine = tok[r * 2:(r + 1) * 2]
            ref(mine[:, :-1], labels=mine[:, 1:]).loss.backward()
            grads.append({n: (p.grad.clone() if p.grad is not None else None) for n, p in ref.named_parameters()})
        for n, p in ref.named_parameters():
            gs = [g[n] for g in grads]
            if all(g is None for g in gs):
                p.grad = None
            else:
                p.grad = sum(g if g is not None else torch.zeros_like(p) for g in gs) / world
        torch.nn.utils.clip_grad_norm_([p for p in ref.parameters() if p.grad is not None], 1.0)
        opt.step()
        opt.zero_grad(set_to_none=True)
    sd = ref.state_dict()
    for k, v in got.items():
        torch.testing.assert_close(v, sd[k], rtol=1e-4, atol=1e-5, msg=k)
    torch.testing.assert_close(got["layers.1.never.weight"], init_never, rtol=0, atol=0)


def _order_worker(rank, world, out):
    from parallel_b200.models.config import resolve_config
    from parallel_b200.models.qwen3 import build_model
    from parallel_b200.parallel.engine import ParallelEngine
    from parallel_b200.parallel.param_unit import DPParamUnit
    from parallel_b200.state import ParallelConfig

    events = []
    orig_reduce, orig_finish = DPParamUnit.reduce_gradients, DPParamUnit.finish_gradient_reduction

    def reduce(self, grads):
        events.append(("start", self.unit_index, sum(u.reduction_in_flight for u in units) + 1))
        return orig_reduce(self, grads)

    def finish(self):
        if self.reduction_in_flight:
            events.append(("finish", self.unit_index, None))
        return orig_finish(self)

    DPParamUnit.reduce_gradients, DPParamUnit.finish_gradient_reduction = reduce, finish
    cfg = cpu_cfg(**{"parallel.dp_shard": world, "engine.overlap_backward_reductions": "true"})
    pc = ParallelConfig(cfg)
    pc.set_device_mesh("cpu")
    cfg_m = resolve_config("tiny-qwen3", num_hidden_layers=4)
    m = build_model(cfg_m, dtype=torch.float32, seed=0)
    eng = ParallelEngine(m, None, pc, cfg, torch.device("cpu"))
    units = eng.fsdp_wrapper.units
    tok = torch.randint(0, 1024, (2, 33), generator=torch.Generator().manual_seed(rank))
    loss = eng.forward(tok[:, :-1], tok[:, 1:]).loss
    eng.backward(loss)
    if rank == 0:
        torch.save(events, out)


def test_fsdp_reductions_reverse_order_at_most_two_in_flight(tmp_path):
    """Overlapped backward: every unit's reduce-scatter starts in strict reverse
    unit order (layers last-to-first, then the root unit at the end), with at
    most two in flight, and each is drained before the backward returns (the
    reference's schedule, dp_sharded.py:305-321)."""
    out = str(tmp_path / "order.pt")
    run_ranks(_order_worker, 2, out)
    events = torch.load(out, weights_only=False)
    starts = [u for kind, u, _ in events if kind == "start"]
    assert starts == [4, 3, 2, 1, 0], events  # unit 0 = root (embedding, final norm), 1..4 = layers
    assert max(n for kind, _, n in events if kind == "start") <= 2, events
    assert sorted(u for kind, u, _ in events if kind == "finish") == [0, 1, 2, 3, 4], events


def _collective_count_worker(rank, world, ckpt, out):
    import torch.distributed as dist

    from parallel_b200.models.config import resolve_config
    from parallel_b200.models.qwen3 import build_model
    from parallel_b200.parallel.engine import ParallelEngine
    from parallel_b200.state import ParallelConfig

    calls = {"all_gather": [], "reduce_scatter": []}
    real_ag, real_rs = dist.all_gather_into_tensor, dist.reduce_scatter_tensor

    def ag(*a, **k):
        calls["all_gather"].append(a[1].numel())
        return real_ag(*a, **k)

    def rs(*a, **k):
        calls["reduce_scatter"].append(a[1].numel())
        return real_rs(*a, **k)

    cfg = cpu_cfg(**{"parallel.dp_shard": world, "engine.activation_checkpoint": str(ckpt).lower()})
    pc = ParallelConfig(cfg)
    pc.set_device_mesh("cpu")
    m = build_model(resolve_config("tiny-qwen3"), dtype=torch.float32, seed=0)
    eng = ParallelEngine(m, None, pc, cfg, torch.device("cpu"))
    buckets = [u.bucket_numel for u in eng.fsdp_wrapper.units]
    tok = torch.randint(0, 1024, (2, 33), generator=torch.Generator().manual_seed(rank))
    dist.all_gather_into_tensor, dist.reduce_scatter_tensor = ag, rs
    try:
        loss = eng.forward(tok[:, :-1], tok[:, 1:]).loss
        eng.backward(loss)
    finally:
        dist.all_gather_into_tensor, dist.reduce_scatter_tensor = real_ag, real_rs
    if rank == 0:
        torch.save({"calls": calls, "buckets": buckets}, out)


@pytest.mark.parametrize("ckpt", [False, True])
def test_fsdp_one_packed_collective_per_unit_each_way(tmp_path, ckpt):
    """Every unit moves its whole flat bucket in ONE all-gather per gather and
    ONE reduce-scatter per backward: the root unit (embedding, final norm) is
    gathered once and kept; each layer is gathered for the forward and again
    for its backward (resharded in between)."""
    out = str(tmp_path / "calls.pt")
    run_ranks(_collective_count_worker, 2, ckpt, out)
    got = torch.load(out, weights_only=False)
    buckets, calls = got["buckets"], got["calls"]
    root, layers = buckets[0], buckets[1:]
    assert sorted(calls["all_gather"]) == sorted([root] + 2 * layers), calls
    assert sorted(calls["reduce_scatter"]) == sorted(2 * b for b in buckets), calls


def _buffer_worker(rank, world, out_q):
    from parallel_b200.models.config import resolve_config
    from parallel_b200.models.qwen3 import build_model
    from parallel_b200.parallel.engine import ParallelEngine
    from parallel_b200.state import ParallelConfig

    cfg = cpu_cfg(**{"parallel.dp_replicate": 2, "parallel.dp_shard": 2})
    pc = ParallelConfig(cfg)
    pc.set_device_mesh("cpu")
    m = build_model(resolve_config("tiny-qwen3"), dtype=torch.float32, seed=0)
    eng = ParallelEngine(m, None, pc, cfg, torch.device("cpu"))
    buf = m.model.rotary_emb.inv_freq
    buf.add_(float(rank))  # diverge on purpose
    eng.sync_buffers()
    got = [torch.zeros_like(buf) for _ in range(world)]
    import torch.distributed as dist

    dist.all_gather(got, buf.contiguous())
    if rank == 0:
        torch.save(got, out_q)


def test_sync_buffers_broadcasts_from_the_first_replica_and_shard(tmp_path):
    """sync_buffers (before eval) makes every rank's buffers equal to global
    rank 0's, over the replicate and the shard groups."""
    out = str(tmp_path / "buf.pt")
    run_ranks(_buffer_worker, 4, out)
    got = torch.load(out, weights_only=False)
    for g in got[1:]:
        torch.testing.assert_close(g, got[0], rtol=0, atol=0)


def _strict_worker(rank, world, out_q):
    from parallel_b200.models.config import resolve_config
    from parallel_b200.models.qwen3 import build_model
    from parallel_b200.parallel.engine import ParallelEngine
    from parallel_b200.state import ParallelConfig

    cfg = cpu_cfg(**{"parallel.dp_shard": 2})
    pc = ParallelConfig(cfg)
    pc.set_device_mesh("cpu")
    src = build_model(resolve_config("tiny-qwen3"), dtype=torch.float32, seed=3).state_dict()
    m = build_model(resolve_config("tiny-qwen3"), dtype=torch.float32, seed=0)
    eng = ParallelEngine(m, None, pc, cfg, torch.device("cpu"))
    partial = {k: v for k, v in src.items() if k != "model.norm.weight"}
    strict_error = None
    try:
        eng.load_state_dict(partial)
    except RuntimeError as e:
        strict_error = str(e)
    eng.load_state_dict(partial, strict=False)
    full = eng.state_dict()
    if rank == 0:
        torch.save({"err": strict_error, "full": full, "src": src}, out_q)


def test_load_state_dict_strictness_on_every_rank(tmp_path):
    """A portable state dict missing a key is rejected with strict=True (on
    every rank: no rank is left half-loaded) and loads the rest with
    strict=False."""
    out = str(tmp_path / "strict.pt")
    run_ranks(_strict_worker, 2, out)
    got = torch.load(out, weights_only=False)
    assert got["err"] is not None and "model.norm.weight" in got["err"], got["err"]
    for k, v in got["src"].items():
        if k != "model.norm.weight":
            torch.testing.assert_close(got["full"][k], v, rtol=0, atol=0, msg=k)
