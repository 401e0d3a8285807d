"""Multi-GPU training against a single-process oracle.

Each case trains a small model for two AdamW steps on 2 or 4 GPUs (bf16, the
default NVLink / fused data plane, activation checkpointing on) and compares
the logged losses, the global gradient norms and the full model after the
steps with a single-process fp32 run of the same model on the same global
batch (CPU, plain PyTorch).  It then checks the exact-topology checkpoint:
an engine restored from it takes the same next step as the original.
Tolerances are the reference's GPU-test tolerances (loss 5e-2 / 5e-3,
parameters 5e-2 / 5e-3, gradient norm 2e-2 relative;
``tests/gpu/test_distributed_gpu.py`` of the reference).  The MoE model's
router weights are scaled so that bf16 rounding cannot flip a near-tie top-k
routing decision between the bf16 GPU run and the fp32 oracle.

The graph cases replay the whole model-parallel step as one CUDA graph and
compare it with eager steps of the same engine configuration."""
import os
import subprocess
import sys

import pytest
import torch

pytestmark = pytest.mark.gpu
HERE = os.path.dirname(os.path.abspath(__file__))


def _save_model(path, name):
    from parallel_b200.models.config import resolve_config
    from parallel_b200.models.loading import save_pretrained
    from parallel_b200.models.qwen3 import build_model

    cfg = resolve_config(name)
    m = build_model(cfg, dtype=torch.float32, seed=0)
    with torch.no_grad():
        for n, p in m.named_parameters():
            if n.endswith("mlp.gate.weight"):
                p.mul_(30.0)
    save_pretrained(m, path)


def _oracle(path, batches, dp, model_parallel):
    """Single-process fp32 training with the loss convention of the engine:
    unshifted labels plus the router aux loss on the model-parallel path,
    HF's shifted labels otherwise; data-parallel micro-batches averaged."""
    from parallel_b200.models.config import ModelConfig
    from parallel_b200.models.loading import read_state_dict
    from parallel_b200.models.qwen3 import build_model
    from parallel_b200.parallel.optim import FusedAdamW

    cfg = ModelConfig.from_pretrained(path)
    m = build_model(cfg, dtype=torch.float32, seed=0)
    m.load_state_dict(read_state_dict(path), strict=False)
    m._layout_fused_weights()
    opt = FusedAdamW(list(m.parameters()), lr=1e-3, betas=(0.9, 0.999), weight_decay=0.01)
    losses, norms = [], []
    for tok in batches:
        total = 0.0
        for chunk in tok.chunk(dp, 0):
            x, y = chunk[:, :-1], chunk[:, 1:]
            loss = m(x, labels=y, shift_labels=not model_parallel).loss / dp
            loss.backward()
            total += loss.item()
        norms.append(torch.nn.utils.clip_grad_norm_(list(m.parameters()), 1.0).item())
        opt.step()
        opt.zero_grad(set_to_none=True)
        losses.append(total)
    return losses, norms, m.state_dict()


def _rel(a, b):
    return ((a.float() - b.float()).norm() / (b.float().norm() + 1e-12)).item()


def _run(tmp_path, case, world, overlap="true", port=29600):
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    sys.path.insert(0, HERE)
    import oracle_worker as W

    name, layout = W.CASES[case]
    _save_model(str(tmp_path / "model"), name)
    env = dict(os.environ, PB_ORACLE_CASE=case, PB_ORACLE_TMP=str(tmp_path), PB_ORACLE_OVERLAP=overlap,
               NCCL_NVLS_ENABLE="0")
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nproc-per-node", str(world), "--master-addr",
           "127.0.0.1", "--master-port", str(port), os.path.join(HERE, "oracle_worker.py")]
    subprocess.run(cmd, env=env, check=True, timeout=900)
    res = torch.load(tmp_path / "result.pt", weights_only=False)
    par = layout(world)
    batches = W.data(world, res["dp"])
    losses, norms, state = _oracle(str(tmp_path / "model"), batches, res["dp"], par.get("tp", 1) > 1)
    torch.testing.assert_close(torch.tensor(res["losses"]), torch.tensor(losses), rtol=5e-2, atol=5e-3)
    torch.testing.assert_close(torch.tensor(res["norms"]), torch.tensor(norms), rtol=2e-2, atol=2e-3)
    worst = max(_rel(res["state"][k], v) for k, v in state.items())
    assert worst < 5e-2, worst
    for k, v in state.items():
        torch.testing.assert_close(res["state"][k].float(), v, rtol=5e-2, atol=5e-3)
    # the engine restored from the exact-topology checkpoint takes the original's next step
    a, b = res["cont"]
    assert abs(a - b) <= 1e-3 * max(1.0, abs(a)), res["cont"]
    for k, v in res["after"][0].items():
        assert _rel(res["after"][1][k], v) < 1e-3, k


def test_fsdp_2gpu_matches_single_process(tmp_path):
    _run(tmp_path, "fsdp", 2, port=29601)


def test_fsdp_4gpu_matches_single_process(tmp_path):
    _run(tmp_path, "fsdp", 4, port=29602)


def test_dp_replicate_2gpu_matches_single_process(tmp_path):
    """Replicated data parallelism: the gradient mean over NVLink peer memory."""
    _run(tmp_path, "dp_replicate", 2, port=29608)


def test_hsdp_4gpu_matches_single_process(tmp_path):
    """dp_replicate = 2 x dp_shard = 2: FSDP reduce-scatter, then the replica
    mean of the gradient shards over NVLink peer memory."""
    _run(tmp_path, "hsdp", 4, port=29609)


def test_tp_sp_2gpu_matches_single_process(tmp_path):
    _run(tmp_path, "tp_sp", 2, port=29603)


@pytest.mark.parametrize("overlap", ["true", "false"])
def test_moe_tp_ep_sp_fsdp_4gpu_matches_single_process(tmp_path, overlap):
    _run(tmp_path, "moe_tp_ep_sp_fsdp", 4, overlap=overlap, port=29604 if overlap == "true" else 29605)


def _graph_run(tmp_path, case, world, port):
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    sys.path.insert(0, HERE)
    import oracle_worker as W

    _save_model(str(tmp_path / "model"), W.CASES[case][0])
    env = dict(os.environ, PB_ORACLE_CASE=case, PB_ORACLE_TMP=str(tmp_path), PB_ORACLE_GRAPH="1",
               NCCL_NVLS_ENABLE="0")
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nproc-per-node", str(world), "--master-addr",
           "127.0.0.1", "--master-port", str(port), os.path.join(HERE, "oracle_worker.py")]
    subprocess.run(cmd, env=env, check=True, timeout=900)
    runs = torch.load(tmp_path / "graph_result.pt", weights_only=False)
    (l_e, s_e, _), (l_g, s_g, captured) = runs["eager"], runs["graph"]
    assert captured, "the graph engine never captured its step"
    torch.testing.assert_close(torch.tensor(l_g), torch.tensor(l_e), rtol=2e-3, atol=2e-3)
    worst = max(_rel(s_g[k], v) for k, v in s_e.items())
    assert worst < 1e-2, worst


def test_tp_sp_graph_step_matches_eager_2gpu(tmp_path):
    """Model parallelism (TP = SP = 2, NVLink kernels) replayed as one CUDA graph."""
    _graph_run(tmp_path, "tp_sp", 2, port=29606)


def test_moe_tp_ep_sp_fsdp_graph_step_matches_eager_4gpu(tmp_path):
    """TP + EP + SP over FSDP with the device-resident MoE routing, replayed as
    one CUDA graph with different routings per step."""
    _graph_run(tmp_path, "moe_tp_ep_sp_fsdp", 4, port=29607)
