"""Selection of the in-switch (NVLS) all-reduce on the host: the ``PB_NVLS``
modes and the capability probe, which turns it down on anything but CUDA
devices with switch multicast (the kernel itself is covered by the 2-GPU test
in ``test_multigpu.py``)."""
import os
import tempfile

import pytest
import torch.distributed as dist
import torch

from parallel_b200.parallel.comm.p2p import NvlsAllReduce, ReplicaMeanAllReduce, nvls_mode


@pytest.fixture(scope="module")
def one_rank_group():
    if dist.is_initialized():
        yield dist.group.WORLD
        return
    path = tempfile.mktemp()
    dist.init_process_group("gloo", init_method=f"file://{path}", rank=0, world_size=1)
    yield dist.group.WORLD
    dist.destroy_process_group()


def test_default_mode_is_auto(monkeypatch):
    monkeypatch.delenv("PB_NVLS", raising=False)
    assert nvls_mode() == "auto"


@pytest.mark.parametrize("mode", ["0", "1", "auto"])
def test_probe_declines_on_cpu_groups(one_rank_group, monkeypatch, mode):
    monkeypatch.setenv("PB_NVLS", mode)
    assert NvlsAllReduce.get(one_rank_group, torch.device("cpu"), 1024, force=True) is None


def test_auto_mode_leaves_two_rank_groups_on_peer_loads(monkeypatch):
    """At two ranks both schemes receive the same bytes, so ``auto`` returns
    None before any collective (no process group traffic needed)."""
    monkeypatch.setenv("PB_NVLS", "auto")

    class Two:
        pass

    monkeypatch.setattr(dist, "get_world_size", lambda group=None: 2)
    assert NvlsAllReduce.get(Two(), torch.device("cuda", 0), 1024) is None


def test_replica_mean_needs_cuda_buffers(one_rank_group):
    assert ReplicaMeanAllReduce.get(one_rank_group, torch.device("cpu"), [torch.zeros(8, dtype=torch.bfloat16)]) is None
