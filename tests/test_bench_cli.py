"""Host side of the benchmark script: the configuration it builds for each
benchmark layout and the parallelism name it reports in its JSON line
(names as in the benchmark table: dp_shardN, tp4_sp4_dp_shard2,
tp4_sp4_ep4_dp_shard2).  No GPU needed."""
import os
import sys

import pytest

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
import bench  # noqa: E402


def _args(argv):
    saved = sys.argv
    sys.argv = ["bench.py"] + argv
    try:
        return bench.parse()
    finally:
        sys.argv = saved


@pytest.mark.parametrize("argv,world,name", [
    ([], 1, "single"),
    (["--gpus", "8"], 8, "dp_shard8"),
    (["--gpus", "8", "--model", "Qwen/Qwen3-8B", "--tp", "4", "--sp", "--batch", "1", "--seq", "4096"], 8,
     "tp4_sp4_dp_shard2"),
    (["--gpus", "8", "--model", "Qwen/Qwen3-30B-A3B", "--tp", "4", "--sp", "--ep", "--batch", "1", "--seq", "4096"],
     8, "tp4_sp4_ep4_dp_shard2"),
    (["--gpus", "4", "--tp", "4"], 4, "tp4"),
])
def test_parallelism_names(argv, world, name):
    assert bench.parallelism_name(_args(argv), world) == name


def test_headline_config_matches_the_benchmark_table():
    """Qwen3-0.6B, per-device batch 4 x 2048 tokens, activation checkpointing
    and overlapped reductions on, dp_shard = N."""
    a = _args(["--gpus", "8"])
    assert (a.steps, a.warmup, a.gpus) == (10, 3, 8)
    cfg = bench.make_cfg(a, 8)
    assert cfg.model.name == "Qwen/Qwen3-0.6B"
    assert (cfg.model.per_device_batch_size, cfg.model.max_seq_length) == (4, 2048)
    assert cfg.engine.activation_checkpoint and cfg.engine.overlap_backward_reductions
    assert cfg.parallel.dp_shard == 8 and cfg.data.synthetic


def test_model_parallel_config_folds_sp_and_ep_onto_tp():
    a = _args(["--gpus", "8", "--model", "Qwen/Qwen3-30B-A3B", "--tp", "4", "--sp", "--ep", "--batch", "1",
               "--seq", "4096"])
    cfg = bench.make_cfg(a, 8)
    assert (cfg.parallel.tp, cfg.parallel.sp, cfg.parallel.ep, cfg.parallel.dp_shard) == (4, 4, 4, 2)
    assert (cfg.model.per_device_batch_size, cfg.model.max_seq_length) == (1, 4096)
