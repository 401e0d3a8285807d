"""Host-side pieces of the engine that need no GPU: the whole-step API, the
CUDA-graph refusals and the optimizer step-count bookkeeping of graph replays."""
import pytest
import torch

from dist_utils import cpu_cfg


def _engine():
    from parallel_b200.models.config import resolve_config
    from parallel_b200.models.qwen3 import build_model
    from parallel_b200.parallel.engine import ParallelEngine
    from parallel_b200.state import ParallelConfig

    cfg = cpu_cfg()
    pc = ParallelConfig(cfg)
    pc.set_device_mesh("cpu")
    m = build_model(resolve_config("tiny-qwen3"), dtype=torch.float32, seed=0)
    return ParallelEngine(m, None, pc, cfg, torch.device("cpu")), m


def test_train_step_equals_forward_backward_step():
    a, ma = _engine()
    b, mb = _engine()
    tok = torch.randint(0, 1024, (2, 33), generator=torch.Generator().manual_seed(1))
    la = a.train_step(tok[:, :-1], tok[:, 1:])
    out = b.forward(tok[:, :-1], tok[:, 1:])
    b.backward(out.loss)
    b.step()
    assert abs(float(la) - float(out.loss.detach())) < 1e-6
    for (n, p), q in zip(ma.named_parameters(), mb.parameters()):
        torch.testing.assert_close(p, q, rtol=0, atol=0, msg=n)


def test_train_step_accumulates_stacked_micro_batches():
    """train_step on [A, B, S] equals the training loop's accumulation: each
    micro-batch loss scaled by 1/A, backward per micro-batch, one step."""
    a, ma = _engine()
    b, mb = _engine()
    tok = torch.randint(0, 1024, (3, 2, 33), generator=torch.Generator().manual_seed(2))
    la = a.train_step(tok[..., :-1], tok[..., 1:])
    total = 0.0
    for i in range(3):
        loss = b.forward(tok[i, :, :-1], tok[i, :, 1:]).loss / 3
        b.backward(loss)
        total += float(loss.detach())
    b.step()
    assert abs(float(la) - total) < 1e-6
    for (n, p), q in zip(ma.named_parameters(), mb.parameters()):
        torch.testing.assert_close(p, q, rtol=0, atol=0, msg=n)


def test_graph_capture_accepts_moe_models_and_needs_cuda():
    """MoE routing is device-resident, so an MoE engine is not refused for
    being MoE; on a CPU device the capture is refused for the device."""
    from parallel_b200.models.config import resolve_config
    from parallel_b200.models.qwen3 import build_model
    from parallel_b200.parallel.engine import ParallelEngine
    from parallel_b200.parallel.graph_step import capture_unsupported
    from parallel_b200.state import ParallelConfig

    cfg = cpu_cfg()
    pc = ParallelConfig(cfg)
    pc.set_device_mesh("cpu")
    m = build_model(resolve_config("tiny-qwen3-moe"), dtype=torch.float32, seed=0)
    eng = ParallelEngine(m, None, pc, cfg, torch.device("cpu"))
    assert capture_unsupported(eng) is None
    with pytest.raises(NotImplementedError, match="CUDA device"):
        eng.enable_graph_capture()
    assert eng._graph_pending is None


def test_graph_capture_refused_on_cpu():
    eng, _ = _engine()
    tok = torch.randint(0, 1024, (2, 17))
    with pytest.raises(RuntimeError, match="CUDA"):
        eng.capture_train_step(tok[:, :-1], tok[:, 1:])
    assert eng._graph is None


def test_graph_step_count_bookkeeping():
    """A capture advances the host step counters without running: they are
    restored afterwards; each replay advances them once."""
    from parallel_b200.parallel.optim import FusedAdamW

    p = torch.nn.Parameter(torch.randn(8))
    opt = FusedAdamW([p], lr=1e-2)
    p.grad = torch.randn(8)
    opt.step()
    counts = opt.graph_step_counts()
    assert float(counts[id(p)]) == 1.0
    opt.state[p]["step"] += 1  # what a capture does on the host
    opt.restore_step_counts(counts)
    assert float(opt.state[p]["step"]) == 1.0


def test_capture_unsupported_names_each_host_side_decision():
    from types import SimpleNamespace as NS

    from parallel_b200.parallel.graph_step import capture_unsupported

    def eng(moe=False, mp=False, scaler=False, fsdp=True, offload=False, unused=False, rep=1, fused=True,
            experts=128):
        opt = NS(enable_graph_hyper=lambda d: None) if fused else NS()
        return NS(model=NS(config=NS(is_moe=moe, num_experts=experts, hidden_size=2048)), mp_wrapper=NS(is_active=mp),
                  grad_scaler=NS(is_enabled=lambda: scaler),
                  fsdp_wrapper=NS(is_active=fsdp, cpu_offload=offload, find_unused_parameters=unused),
                  pconfig=NS(dp_replicate_size=rep), optimizer=opt)

    assert capture_unsupported(eng()) is None
    assert capture_unsupported(eng(fsdp=True, rep=2)) is None          # hybrid: bucket all-reduce, capturable
    assert capture_unsupported(eng(fsdp=False)) is None                 # single device
    assert capture_unsupported(eng(moe=True)) is None                   # device-resident routing
    assert "MoE" in capture_unsupported(eng(moe=True, experts=512))
    assert capture_unsupported(eng(mp=True)) is None                    # NVLink TP / SP / EP
    nccl_ep = eng(mp=True)
    nccl_ep.mp_wrapper.expert_runtime = NS(dispatcher=object(), transport=None)
    assert "all-to-all" in capture_unsupported(nccl_ep)
    assert "fp16" in capture_unsupported(eng(scaler=True))
    assert "cpu_offload" in capture_unsupported(eng(offload=True))
    assert "find_unused" in capture_unsupported(eng(unused=True))
    assert "DP-replicate" in capture_unsupported(eng(fsdp=False, rep=2))
    assert "FusedAdamW" in capture_unsupported(eng(fused=False))


def test_fp16_loss_scaling_halves_the_scale_on_non_finite_gradients():
    """config.amp_dtype=fp16: the GradScaler path (the reference's
    engine.py:201-221 semantics): a non-finite step leaves the parameters
    untouched and halves the scale instead of raising; finite steps update."""
    from parallel_b200.models.config import resolve_config
    from parallel_b200.models.qwen3 import build_model
    from parallel_b200.parallel.engine import ParallelEngine
    from parallel_b200.state import ParallelConfig

    cfg = cpu_cfg(**{"config.use_amp": "true", "config.amp_dtype": "fp16"})
    pc = ParallelConfig(cfg)
    pc.set_device_mesh("cpu")
    m = build_model(resolve_config("tiny-qwen3"), dtype=torch.float32, seed=0)
    eng = ParallelEngine(m, None, pc, cfg, torch.device("cpu"))
    assert eng.grad_scaler.is_enabled()
    tok = torch.randint(0, 1024, (2, 33), generator=torch.Generator().manual_seed(4))
    before = {n: p.detach().clone() for n, p in m.named_parameters()}
    eng.backward(eng.forward(tok[:, :-1], tok[:, 1:]).loss)
    next(p for p in m.parameters() if p.grad is not None).grad.view(-1)[0] = float("inf")
    scale = eng.grad_scaler.get_scale()
    eng.step()                                     # no FloatingPointError with a scaler
    assert eng.grad_scaler.get_scale() == scale / 2
    for n, p in m.named_parameters():
        torch.testing.assert_close(p.detach(), before[n], rtol=0, atol=0, msg=n)
        assert p.grad is None
    eng.backward(eng.forward(tok[:, :-1], tok[:, 1:]).loss)
    eng.step()
    assert any(not torch.equal(p.detach(), before[n]) for n, p in m.named_parameters())
