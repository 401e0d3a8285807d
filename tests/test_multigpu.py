"""Multi-GPU tests (NVLink P2P collectives vs NCCL) and the bounded-wait status path."""
import json
import os
import subprocess
import sys

import pytest
import torch

pytestmark = pytest.mark.gpu
HERE = os.path.dirname(os.path.abspath(__file__))


def test_bounded_wait_times_out_and_context_survives():
    from parallel_b200.ops._ext import ext

    C = ext()
    flag = torch.zeros(1, dtype=torch.int32, device="cuda")   # nothing ever sets it
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    C.wait_flag(flag, 1, 0.5, status)
    torch.cuda.synchronize()
    assert int(status.item()) == 2  # kErrPeerTimeout
    a = torch.randn(256, 256, device="cuda").to(torch.bfloat16)
    out = torch.empty(256, 256, device="cuda", dtype=torch.bfloat16)
    C.gemm(a, a, out, False, False, 0, 1.0)
    torch.cuda.synchronize()
    assert torch.isfinite(out.float()).all()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_fsdp_p2p_collectives_match_nccl(tmp_path):
    out = tmp_path / "res.json"
    env = dict(os.environ, PB_TEST_OUT=str(out), NCCL_NVLS_ENABLE="0")
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nproc-per-node", "2", "--master-addr", "127.0.0.1",
           "--master-port", "29533", os.path.join(HERE, "multigpu_worker.py")]
    subprocess.run(cmd, env=env, check=True, timeout=600)
    res = json.loads(out.read_text())
    assert res["names"] == ["p2p", "nccl"]
    for a, b in zip(res["p2p"], res["nccl"]):
        assert abs(a - b) < 2e-2 * max(1.0, abs(b)), res
    assert res["state_rel_diff"] < 2e-2, res


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
@pytest.mark.parametrize("sp_mode", ["pull", "fused"])
def test_fused_sequence_parallel_matches_nccl(tmp_path, sp_mode):
    """tp = sp = 2: the NVLink sequence-parallel data plane (pull: peer gather
    + GEMM and GEMM + owner-pull reduce; fused: all-gather inside the
    column-parallel GEMMs, reduce-scatter inside the row-parallel GEMMs) gives
    the same losses and gradients as the NCCL sequence-parallel path."""
    out = tmp_path / "res_sp.json"
    env = dict(os.environ, PB_TEST_OUT=str(out), PB_TEST_MODE="sp", PB_TEST_TMP=str(tmp_path), NCCL_NVLS_ENABLE="0",
               PB_SP_MODE=sp_mode)
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nproc-per-node", "2", "--master-addr", "127.0.0.1",
           "--master-port", "29534", os.path.join(HERE, "multigpu_worker.py")]
    subprocess.run(cmd, env=env, check=True, timeout=600)
    res = json.loads(out.read_text())
    assert res["used_fused"] == [True, False], res
    for a, b in zip(res["fused"], res["nccl"]):
        assert abs(a - b) < 2e-2 * max(1.0, abs(b)), res
    assert res["grad_rel_diff"] < 3e-2, res


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_p2p_expert_dispatch_matches_nccl(tmp_path):
    """Qwen3-MoE with tp = sp = ep = 2: token dispatch / combine over NVLink peer
    memory give the same losses and gradients as the NCCL all-to-all path."""
    out = tmp_path / "res_moe.json"
    env = dict(os.environ, PB_TEST_OUT=str(out), PB_TEST_MODE="sp", PB_TEST_MOE="1", PB_TEST_TMP=str(tmp_path),
               NCCL_NVLS_ENABLE="0")
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nproc-per-node", "2", "--master-addr", "127.0.0.1",
           "--master-port", "29535", os.path.join(HERE, "multigpu_worker.py")]
    subprocess.run(cmd, env=env, check=True, timeout=600)
    res = json.loads(out.read_text())
    assert res["used_fused"] == [True, False], res
    for a, b in zip(res["fused"], res["nccl"]):
        assert abs(a - b) < 2e-2 * max(1.0, abs(b)), res
    assert res["grad_rel_diff"] < 5e-2, res


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_p2p_small_all_reduce_matches_nccl(tmp_path):
    """Peer-memory small all-reduce (sum, max, log-sum-exp merge) equals NCCL,
    across sizes and inside a replayed CUDA graph."""
    out = tmp_path / "res_small.json"
    env = dict(os.environ, PB_TEST_OUT=str(out), PB_TEST_MODE="small", NCCL_NVLS_ENABLE="0")
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nproc-per-node", "2", "--master-addr", "127.0.0.1",
           "--master-port", "29536", os.path.join(HERE, "multigpu_worker.py")]
    subprocess.run(cmd, env=env, check=True, timeout=600)
    res = json.loads(out.read_text())
    assert res["worst"] < 1e-5, res


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
@pytest.mark.parametrize("moe", ["0", "1"])
def test_fused_tensor_parallel_matches_nccl(tmp_path, moe):
    """tp = 2 without sequence parallelism: GEMM -> all-reduce over NVLink for
    the row-parallel outputs and the column-parallel input gradients, the
    embedding all-reduce and (MoE) the replicated-token expert all-reduces on
    peer memory give the NCCL path's losses and gradients."""
    out = tmp_path / "res_tp.json"
    env = dict(os.environ, PB_TEST_OUT=str(out), PB_TEST_MODE="sp", PB_TEST_SP="0", PB_TEST_MOE=moe,
               PB_TEST_TMP=str(tmp_path), NCCL_NVLS_ENABLE="0")
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nproc-per-node", "2", "--master-addr", "127.0.0.1",
           "--master-port", "29537", os.path.join(HERE, "multigpu_worker.py")]
    subprocess.run(cmd, env=env, check=True, timeout=600)
    res = json.loads(out.read_text())
    assert res["used_fused"] == [True, False], res
    for a, b in zip(res["fused"], res["nccl"]):
        assert abs(a - b) < 2e-2 * max(1.0, abs(b)), res
    assert res["grad_rel_diff"] < 3e-2, res


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_nvls_all_reduce_matches_fp32_sum(tmp_path):
    """In-switch all-reduce (multimem.ld_reduce + multimem.st over the
    multicast address of the symmetric buffer) equals an fp32 sum of the same
    bf16 inputs rounded once; also through the replicate-mean wrapper and in a
    replayed CUDA graph.  Skips where the fabric offers no switch multicast."""
    out = tmp_path / "res_nvls.json"
    env = dict(os.environ, PB_TEST_OUT=str(out), PB_TEST_MODE="nvls", PB_NVLS="1")
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nproc-per-node", "2", "--master-addr", "127.0.0.1",
           "--master-port", "29538", os.path.join(HERE, "multigpu_worker.py")]
    subprocess.run(cmd, env=env, check=True, timeout=600)
    res = json.loads(out.read_text())
    if "skipped" in res:
        pytest.skip(res["skipped"])
    assert res["replica_uses_nvls"], res
    assert res["worst"] < 8e-3, res
