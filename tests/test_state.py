"""Topology validation, mesh layout and RNG policy (CPU, no process group)."""
import pytest
import torch

from parallel_b200.config import Config
from parallel_b200.state import ParallelConfig, RuntimeState, Strategies, reset_runtime_state


def _config(**overrides):
    par = {"dp_replicate": 1, "dp_shard": 1, "tp": 1, "cp": 1, "sp": 1, "ep": 1, "pp": 1}
    par.update(overrides)
    return Config({"parallel": par})


def _fake_world(monkeypatch, n):
    monkeypatch.setenv("WORLD_SIZE", str(n))
    monkeypatch.setattr("parallel_b200.state.is_dist_initialized", lambda: True)
    monkeypatch.setattr("parallel_b200.state.dist.get_rank", lambda: 0)
    monkeypatch.setattr("parallel_b200.state.dist.get_world_size", lambda: n)


def test_runtime_state_defaults_to_single_process(monkeypatch):
    monkeypatch.delenv("WORLD_SIZE", raising=False)
    reset_runtime_state()
    env = RuntimeState()
    assert env.world_size == 1 and env.rank == 0 and env.can_log
    assert RuntimeState(backend="nccl") is env  # fixed by the first call
    reset_runtime_state()


def test_rejects_mesh_world_size_mismatch():
    with pytest.raises(ValueError, match="does not match"):
        ParallelConfig(_config(dp_shard=2))


def test_rejects_non_positive_dimensions():
    with pytest.raises(ValueError, match="positive integers"):
        ParallelConfig(_config(dp_replicate=0))


def test_tp_mesh_layout_and_strides(monkeypatch):
    _fake_world(monkeypatch, 8)
    c = ParallelConfig(_config(tp=4, ep=4, dp_shard=2))
    assert c.get_mesh_layout() == ((Strategies.DP_REPLICATE, Strategies.TP, Strategies.DP_SHARD), (1, 4, 2), (8, 1, 4))
    assert c.get_mesh_dims() == ((Strategies.TP, Strategies.DP_SHARD), (4, 2))
    assert c.model_parallel_size == 4 and c.total_size == 8


def test_sequence_parallel_folds_onto_tp(monkeypatch):
    _fake_world(monkeypatch, 8)
    c = ParallelConfig(_config(tp=4, sp=4, ep=4, dp_shard=2))
    assert c.total_size == 8
    assert Strategies.SP not in c.get_mesh_layout()[0]
    with pytest.raises(ValueError, match="sp == 1 or sp == tp"):
        ParallelConfig(_config(tp=4, sp=2, ep=4, dp_shard=2))


def test_rejects_unfolded_tp_ep(monkeypatch):
    _fake_world(monkeypatch, 8)
    with pytest.raises(ValueError, match="tp == ep"):
        ParallelConfig(_config(tp=4, ep=2, dp_shard=2))


def test_tp_adjacent_physical_mesh(monkeypatch):
    _fake_world(monkeypatch, 8)
    c = ParallelConfig(_config(tp=4, ep=4, dp_shard=2))
    names, shape, strides = c.get_mesh_layout()
    assert c._physical_mesh(names, shape, strides).tolist() == [[[0, 4], [1, 5], [2, 6], [3, 7]]]


def test_dense_tp_without_ep(monkeypatch):
    _fake_world(monkeypatch, 8)
    c = ParallelConfig(_config(tp=4, dp_shard=2))
    assert c.tp_size == 4 and c.ep_size == 1


def test_rejects_context_and_pipeline_parallel(monkeypatch):
    _fake_world(monkeypatch, 2)
    with pytest.raises(NotImplementedError, match="tensor parallel"):
        ParallelConfig(_config(cp=2))
    with pytest.raises(NotImplementedError, match="tensor parallel"):
        ParallelConfig(_config(pp=2))


def test_rejects_expert_tensor_parallel(monkeypatch):
    _fake_world(monkeypatch, 2)
    cfg = _config(tp=2, ep=2)
    cfg.parallel.expert_tp = 2
    with pytest.raises(NotImplementedError, match="expert_tp"):
        ParallelConfig(cfg)


class _FakeMesh:
    mesh_dim_names = ("dp_replicate", "dp_shard")

    def __init__(self, rep, shard):
        self.ranks = {"dp_replicate": rep, "dp_shard": shard}

    def get_local_rank(self, name):
        return self.ranks[name]


def _hybrid(rep=1, shard=2):
    c = ParallelConfig.__new__(ParallelConfig)
    c.dp_replicate_size, c.dp_shard_size = 2, 4
    c.device_mesh = _FakeMesh(rep, shard)
    c.device_type = "cpu"
    c.local_rank = 0
    c._device = None
    return c


def test_data_rank_covers_replicate_and_shard():
    c = _hybrid(1, 2)
    assert c.data_rank == 6
    assert c.data_world_size == 8


def test_training_rng_uses_data_rank(monkeypatch):
    c = _hybrid(1, 2)
    rs, ns, ts = [], [], []
    monkeypatch.setattr("parallel_b200.state.random.seed", rs.append)
    monkeypatch.setattr("parallel_b200.state.np.random.seed", ns.append)
    monkeypatch.setattr("parallel_b200.state.torch.manual_seed", ts.append)
    c.model_train_rngs(seed=10)
    assert rs == [16] and ns == [16] and ts == [6010]


def test_device_property():
    assert _hybrid().device == torch.device("cpu")
