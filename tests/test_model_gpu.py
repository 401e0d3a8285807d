"""The fused CUDA model path against the fp32 PyTorch path of the same model."""
import copy

import pytest
import torch

pytestmark = pytest.mark.gpu


def _pair(name, seed=0):
    from parallel_b200.models.config import resolve_config
    from parallel_b200.models.qwen3 import build_model

    cfg = resolve_config(name)
    ref = build_model(cfg, dtype=torch.float32, seed=seed)
    gpu = build_model(cfg, dtype=torch.bfloat16, seed=seed)
    gpu.load_state_dict({k: v.to(torch.bfloat16) for k, v in ref.state_dict().items()})
    gpu.to("cuda")
    gpu._layout_fused_weights()
    return cfg, ref, gpu


def _rel(a, b):
    return ((a.float() - b.float()).norm() / (b.float().norm() + 1e-12)).item()


def _pin_routing(ref, gpu):
    """Make the fp32 model route every token to the experts the bf16 model
    chose.  bf16 rounding flips near-tie top-k decisions, and a flipped route
    moves a token's whole contribution between experts; with the choices
    pinned the two models compute the same function and only rounding differs.
    The fp32 router still computes its own softmax and routing weights."""
    chosen = []

    def record(module, args, out):
        chosen.append(out[2].detach().cpu())

    hooks = [m.register_forward_hook(record) for n, m in gpu.named_modules() if n.endswith("mlp.gate")]
    routers = [m for n, m in ref.named_modules() if n.endswith("mlp.gate")]

    def pinned(router, i):
        def forward(x):
            x2 = x.reshape(-1, x.shape[-1])
            probs = torch.softmax(torch.nn.functional.linear(x2, router.weight), dim=-1, dtype=torch.float32)
            idx = chosen[i]
            top_v = probs.gather(1, idx)
            if router.norm_topk_prob:
                top_v = top_v / top_v.sum(dim=-1, keepdim=True)
            return probs, top_v, idx

        return forward

    for i, r in enumerate(routers):
        r.forward = pinned(r, i)
    return hooks


@pytest.mark.parametrize("name", ["small-qwen3", "small-qwen3-moe"])
def test_cuda_model_matches_fp32(name):
    cfg, ref, gpu = _pair(name)
    torch.manual_seed(0)
    ids = torch.randint(0, cfg.vocab_size, (2, 256))
    hooks = _pin_routing(ref, gpu) if cfg.is_moe else []
    out_gpu = gpu(ids.cuda(), labels=ids.cuda())  # the bf16 model routes first
    out_ref = ref(ids, labels=ids)
    for h in hooks:
        h.remove()
    # GPU bf16 tolerances of the reference's GPU tests (loss 5e-2 / 5e-3)
    torch.testing.assert_close(out_gpu.loss.float().cpu(), out_ref.loss, rtol=5e-2, atol=5e-3)
    out_ref.loss.backward()
    out_gpu.loss.backward()
    gp = dict(gpu.named_parameters())
    for n, p in ref.named_parameters():
        err = _rel(gp[n].grad.cpu(), p.grad)
        assert err < 8e-2, (n, err)


def test_engine_trains_on_gpu():
    from parallel_b200.config import from_dotlist, load_cfg, merge
    from parallel_b200.ops._ext import check_device_errors
    from parallel_b200.parallel.engine import ParallelEngine
    from parallel_b200.state import ParallelConfig

    cfg, ref, gpu = _pair("small-qwen3")
    c = merge(load_cfg(argv=[]), from_dotlist(["config.device_type=cuda", "model.learning_rate=3e-3"]))
    pc = ParallelConfig(c)
    pc.set_device_mesh("cuda")
    eng = ParallelEngine(gpu, None, pc, c, torch.device("cuda", 0))
    tok = torch.randint(0, cfg.vocab_size, (4, 129), device="cuda")
    losses = []
    for _ in range(8):
        loss = eng.forward(tok[:, :-1], tok[:, 1:]).loss
        eng.backward(loss)
        eng.step()
        losses.append(loss.item())
    torch.cuda.synchronize()
    check_device_errors()
    assert losses[-1] < losses[0] - 0.5, losses
    assert eng.last_grad_norm is not None and torch.isfinite(eng.last_grad_norm).all()


def test_cuda_graph_step_matches_eager():
    """A captured-and-replayed training step follows the eager trajectory
    (same kernels in the same order; lr and bias corrections read from the
    device), including an lr change between replays."""
    from parallel_b200.config import from_dotlist, load_cfg, merge
    from parallel_b200.ops._ext import check_device_errors
    from parallel_b200.parallel.engine import ParallelEngine
    from parallel_b200.state import ParallelConfig

    c = merge(load_cfg(argv=[]), from_dotlist(["config.device_type=cuda", "model.learning_rate=3e-3"]))
    engines = []
    for _ in range(2):
        cfg, _, gpu = _pair("small-qwen3")
        pc = ParallelConfig(c)
        pc.set_device_mesh("cuda")
        engines.append(ParallelEngine(gpu, None, pc, c, torch.device("cuda", 0)))
    eager, graphed = engines
    g = torch.Generator().manual_seed(3)
    toks = [torch.randint(0, cfg.vocab_size, (4, 129), generator=g).cuda() for _ in range(5)]
    # the capture runs its warm-up steps eagerly on the capture batch
    graphed.capture_train_step(toks[0][:, :-1], toks[0][:, 1:], warmup=2)
    for _ in range(2):
        eager.train_step(toks[0][:, :-1], toks[0][:, 1:])
    le, lg = [], []
    for i in range(1, 5):
        if i == 3:
            for e in engines:
                e.optimizer.param_groups[0]["lr"] = 1e-3
        le.append(float(eager.train_step(toks[i][:, :-1], toks[i][:, 1:])))
        lg.append(float(graphed.train_step(toks[i][:, :-1], toks[i][:, 1:])))
    torch.cuda.synchronize()
    check_device_errors()
    assert max(abs(a - b) for a, b in zip(le, lg)) < 2e-2, (le, lg)
    pe, pg = dict(eager.model.named_parameters()), dict(graphed.model.named_parameters())
    for n, p in pe.items():
        assert _rel(pg[n].detach(), p.detach()) < 2e-2, n
    se = eager.optimizer.state[next(iter(eager.optimizer.state))]["step"]
    sg = graphed.optimizer.state[next(iter(graphed.optimizer.state))]["step"]
    assert float(se) == float(sg) == 6.0
    graphed.release_graph()


def test_deferred_graph_capture_follows_the_eager_trajectory():
    """engine.compile's mode: two eager steps on the capture stream, then the
    capture, then replays - each batch trained on exactly once, so the losses
    and weights follow a plain eager run."""
    from parallel_b200.config import from_dotlist, load_cfg, merge
    from parallel_b200.ops._ext import check_device_errors
    from parallel_b200.parallel.engine import ParallelEngine
    from parallel_b200.state import ParallelConfig

    c = merge(load_cfg(argv=[]), from_dotlist(["config.device_type=cuda", "model.learning_rate=3e-3"]))
    engines = []
    for _ in range(2):
        cfg, _, gpu = _pair("small-qwen3")
        pc = ParallelConfig(c)
        pc.set_device_mesh("cuda")
        engines.append(ParallelEngine(gpu, None, pc, c, torch.device("cuda", 0)))
    eager, graphed = engines
    graphed.enable_graph_capture(warmup_steps=2)
    g = torch.Generator().manual_seed(5)
    toks = [torch.randint(0, cfg.vocab_size, (4, 129), generator=g).cuda() for _ in range(6)]
    le, lg = [], []
    for i, t in enumerate(toks):
        le.append(float(eager.train_step(t[:, :-1], t[:, 1:])))
        lg.append(float(graphed.train_step(t[:, :-1], t[:, 1:])))
        assert (graphed._graph is not None) == (i >= 2)
    torch.cuda.synchronize()
    check_device_errors()
    assert max(abs(a - b) for a, b in zip(le, lg)) < 2e-2, (le, lg)
    pe, pg = dict(eager.model.named_parameters()), dict(graphed.model.named_parameters())
    for n, p in pe.items():
        assert _rel(pg[n].detach(), p.detach()) < 2e-2, n
    se = eager.optimizer.state[next(iter(eager.optimizer.state))]["step"]
    sg = graphed.optimizer.state[next(iter(graphed.optimizer.state))]["step"]
    assert float(se) == float(sg) == 6.0
    graphed.release_graph()


def test_graph_step_accumulates_micro_batches():
    """A captured step over two stacked micro-batches [2, B, S] follows the
    eager accumulation (loss / 2 per micro-batch, one optimizer step)."""
    from parallel_b200.config import from_dotlist, load_cfg, merge
    from parallel_b200.ops._ext import check_device_errors
    from parallel_b200.parallel.engine import ParallelEngine
    from parallel_b200.state import ParallelConfig

    c = merge(load_cfg(argv=[]), from_dotlist(["config.device_type=cuda", "model.learning_rate=3e-3"]))
    engines = []
    for _ in range(2):
        cfg, _, gpu = _pair("small-qwen3")
        pc = ParallelConfig(c)
        pc.set_device_mesh("cuda")
        engines.append(ParallelEngine(gpu, None, pc, c, torch.device("cuda", 0)))
    eager, graphed = engines
    graphed.enable_graph_capture(warmup_steps=1)
    g = torch.Generator().manual_seed(7)
    toks = [torch.randint(0, cfg.vocab_size, (2, 2, 129), generator=g).cuda() for _ in range(4)]
    le, lg = [], []
    for t in toks:
        total = 0.0
        for a in range(2):
            loss = eager.forward(t[a, :, :-1], t[a, :, 1:]).loss / 2
            eager.backward(loss)
            total += float(loss.detach())
        eager.step()
        le.append(total)
        lg.append(float(graphed.train_step(t[..., :-1], t[..., 1:])))
    assert graphed._graph is not None
    torch.cuda.synchronize()
    check_device_errors()
    assert max(abs(a - b) for a, b in zip(le, lg)) < 2e-2, (le, lg)
    pe, pg = dict(eager.model.named_parameters()), dict(graphed.model.named_parameters())
    for n, p in pe.items():
        assert _rel(pg[n].detach(), p.detach()) < 2e-2, n
    graphed.release_graph()


def test_device_error_word_surfaces_as_collective_timeout():
    """A bounded device wait that gave up (its error word, written here from the
    host) is read back asynchronously with the step's finite flag and raised at
    the next step as CollectiveTimeout; the word is cleared."""
    from parallel_b200.config import from_dotlist, load_cfg, merge
    from parallel_b200.ops._ext import ext
    from parallel_b200.parallel.comm.p2p import CollectiveTimeout
    from parallel_b200.parallel.engine import ParallelEngine
    from parallel_b200.state import ParallelConfig

    cfg, _, gpu = _pair("small-qwen3")
    c = merge(load_cfg(argv=[]), from_dotlist(["config.device_type=cuda"]))
    pc = ParallelConfig(c)
    pc.set_device_mesh("cuda")
    eng = ParallelEngine(gpu, None, pc, c, torch.device("cuda", 0))
    tok = torch.randint(0, cfg.vocab_size, (2, 65), device="cuda")
    eng.train_step(tok[:, :-1], tok[:, 1:])
    torch.cuda.synchronize()
    ext().set_error_for_test(0, 2)
    eng.train_step(tok[:, :-1], tok[:, 1:])  # its read-back carries the error
    with pytest.raises(CollectiveTimeout):
        eng.train_step(tok[:, :-1], tok[:, 1:])
    assert ext().read_error(0) == 0
    eng.train_step(tok[:, :-1], tok[:, 1:])  # the engine keeps working
    torch.cuda.synchronize()


@pytest.mark.parametrize("name", ["small-qwen3", "small-qwen3-moe"])
def test_training_steps_are_bitwise_reproducible(name):
    """Two engines built from the same weights and fed the same batches end
    bitwise equal: no kernel of the step accumulates floating point in an
    order that varies between runs (ordered split-K, block partials summed in
    block order, rank- and route-ordered reductions)."""
    from parallel_b200.config import from_dotlist, load_cfg, merge
    from parallel_b200.ops._ext import check_device_errors
    from parallel_b200.parallel.engine import ParallelEngine
    from parallel_b200.state import ParallelConfig

    c = merge(load_cfg(argv=[]), from_dotlist(["config.device_type=cuda", "model.learning_rate=3e-3"]))
    g = torch.Generator().manual_seed(5)
    cfg = None
    runs = []
    for _ in range(2):
        cfg, _, gpu = _pair(name)
        if not runs:
            toks = [torch.randint(0, cfg.vocab_size, (4, 257), generator=g).cuda() for _ in range(3)]
        pc = ParallelConfig(c)
        pc.set_device_mesh("cuda")
        eng = ParallelEngine(gpu, None, pc, c, torch.device("cuda", 0))
        losses = [eng.train_step(t[:, :-1], t[:, 1:]).detach().clone() for t in toks]
        torch.cuda.synchronize()
        check_device_errors()
        runs.append((torch.stack(losses), {n: p.detach().clone() for n, p in eng.model.named_parameters()},
                     eng.last_grad_norm.detach().clone()))
    (la, pa, na), (lb, pb, nb) = runs
    assert torch.equal(la, lb), (la, lb)
    assert torch.equal(na, nb), (na, nb)
    for n, p in pa.items():
        assert torch.equal(p, pb[n]), n


def test_mlp_recompute_without_output_gives_the_same_gradients():
    """The activation-checkpoint recompute runs the dense MLP with its output
    unused (the down GEMM is skipped); differentiating through that output
    gives bitwise the gradients of the full forward."""
    from parallel_b200.ops import functional as Fx

    torch.manual_seed(3)
    T, H, I = 512, 256, 512
    x = torch.randn(T, H, device="cuda").to(torch.bfloat16)
    res = torch.randn(T, H, device="cuda").to(torch.bfloat16)
    wg, wu = (0.05 * torch.randn(I, H, device="cuda")).to(torch.bfloat16), (0.05 * torch.randn(I, H, device="cuda")).to(torch.bfloat16)
    wd = (0.05 * torch.randn(H, I, device="cuda")).to(torch.bfloat16)
    gy = torch.randn(T, H, device="cuda").to(torch.bfloat16)
    grads = []
    for unused in (False, True):
        leaves = [t.detach().clone().requires_grad_(True) for t in (x, wg, wu, wd, res)]
        y = Fx.swiglu_mlp(leaves[0], leaves[1], leaves[2], leaves[3], leaves[4], output_unused=unused)
        grads.append(torch.autograd.grad([y], leaves, [gy]))
    torch.cuda.synchronize()
    for a, b in zip(*grads):
        assert torch.equal(a, b)


def test_decoder_layer_recompute_flag_keeps_gradients():
    """A dense decoder layer run as the FSDP unit's activation-checkpoint
    recompute (``_recomputing`` set: the down projection is skipped) gives
    bitwise the input and parameter gradients of a normal run."""
    cfg, _, gpu = _pair("small-qwen3")
    layer = gpu.model.layers[0]
    B, S = 2, 256
    layer._seq = (B, S)
    layer._inv_freq = gpu.model.rotary_emb.inv_freq
    torch.manual_seed(9)
    x = torch.randn(B, S, cfg.hidden_size, device="cuda").to(torch.bfloat16)
    gy = torch.randn_like(x)
    params = [p for p in layer.parameters()]
    grads = []
    for recompute in (False, True):
        layer._recomputing = recompute
        xi = x.detach().requires_grad_(True)
        y = layer(xi)
        grads.append(torch.autograd.grad([y], [xi] + params, [gy], allow_unused=True))
    layer._recomputing = False
    torch.cuda.synchronize()
    for a, b in zip(*grads):
        assert (a is None and b is None) or torch.equal(a, b)
