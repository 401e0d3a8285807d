"""The training entry point end to end on CPU (synthetic data): logging,
checkpoint cadence, and an exact resume of model, optimizer, RNG and data
stream from a saved checkpoint."""
import os
import re
import subprocess
import sys

import pytest
import torch

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _run(tmp, extra):
    env = dict(os.environ, PYTHONPATH=ROOT, WANDB_MODE="disabled")
    args = [sys.executable, "-m", "parallel_b200.train", f"model.name={tmp}/init", "config.device_type=cpu",
            "config.backend=gloo", "config.use_amp=false", "data.synthetic=true", "config.max_steps=4",
            "config.eval_interval=100", "config.eval_steps=1", "config.grad_accum_steps=2",
            "config.checkpoint_interval=2", f"config.checkpoint_dir={tmp}/ckpt", "model.per_device_batch_size=2",
            "model.max_seq_length=32", "model.learning_rate=1e-3"] + extra
    out = subprocess.run(args, env=env, cwd=tmp, capture_output=True, text=True, timeout=300)
    assert out.returncode == 0, out.stderr[-3000:]
    return {int(m.group(1)): float(m.group(2))
            for m in re.finditer(r"step\s+(\d+) \| loss ([0-9.]+)", out.stdout + out.stderr)}


def test_train_cli_checkpoint_and_exact_resume(tmp_path):
    from parallel_b200.models.config import resolve_config
    from parallel_b200.models.loading import save_pretrained
    from parallel_b200.models.qwen3 import build_model

    tmp = str(tmp_path)
    save_pretrained(build_model(resolve_config("tiny-qwen3"), dtype=torch.float32, seed=0), f"{tmp}/init")
    full = _run(tmp, [])
    assert sorted(full) == [1, 2, 3, 4], full
    assert os.path.isdir(f"{tmp}/ckpt/step-00000002") and os.path.isdir(f"{tmp}/ckpt/step-00000004")
    resumed = _run(tmp, [f"config.resume_from={tmp}/ckpt/step-00000002", f"config.checkpoint_dir={tmp}/ckpt2"])
    assert sorted(resumed) == [3, 4], resumed
    for s in (3, 4):
        assert resumed[s] == full[s], (full, resumed)


def _run_fail(tmp, extra):
    env = dict(os.environ, PYTHONPATH=ROOT, WANDB_MODE="disabled")
    args = [sys.executable, "-m", "parallel_b200.train", f"model.name={tmp}/init", "config.device_type=cpu",
            "config.backend=gloo", "config.use_amp=false", "data.synthetic=true", "config.max_steps=1",
            "model.per_device_batch_size=2", "model.max_seq_length=32"] + extra
    out = subprocess.run(args, env=env, cwd=tmp, capture_output=True, text=True, timeout=300)
    assert out.returncode != 0
    return out.stderr


def test_train_cli_compile_selects_the_graph_step_and_refuses_what_it_cannot_capture(tmp_path):
    """engine.compile=true captures the training step as a CUDA graph: it is
    refused on a CPU device, with a clear error."""
    from parallel_b200.models.config import resolve_config
    from parallel_b200.models.loading import save_pretrained
    from parallel_b200.models.qwen3 import build_model

    tmp = str(tmp_path)
    save_pretrained(build_model(resolve_config("tiny-qwen3"), dtype=torch.float32, seed=0), f"{tmp}/init")
    for accum in (1, 2):
        err = _run_fail(tmp, ["engine.compile=true", f"config.grad_accum_steps={accum}"])
        assert "needs a CUDA device" in err, err[-2000:]


def _run_dist(tmp, extra, port):
    env = dict(os.environ, PYTHONPATH=ROOT, WANDB_MODE="disabled")
    args = [sys.executable, "-m", "torch.distributed.run", "--nproc-per-node", "2", "--master-addr", "127.0.0.1",
            "--master-port", str(port), "-m", "parallel_b200.train", f"model.name={tmp}/init",
            "config.device_type=cpu", "config.backend=gloo", "config.use_amp=false", "data.synthetic=true",
            "config.max_steps=4", "config.eval_interval=100", "config.eval_steps=1",
            "config.checkpoint_interval=2", "model.per_device_batch_size=2", "model.max_seq_length=32",
            "model.learning_rate=1e-3"] + extra
    out = subprocess.run(args, env=env, cwd=tmp, capture_output=True, text=True, timeout=300)
    assert out.returncode == 0, out.stderr[-3000:]
    return {int(m.group(1)): float(m.group(2))
            for m in re.finditer(r"step\s+(\d+) \| loss ([0-9.]+)", out.stdout + out.stderr)}


@pytest.mark.parametrize("topo,port", [(["parallel.dp_shard=2"], 29631), (["parallel.tp=2", "parallel.sp=2"], 29641)])
def test_train_cli_two_ranks_checkpoint_and_exact_resume(tmp_path, topo, port):
    """The entry point under torchrun (2 gloo ranks; FSDP, or TP + SP):
    exact-topology checkpoint at step 2, and a resumed run repeats steps 3-4
    exactly."""
    from parallel_b200.models.config import resolve_config
    from parallel_b200.models.loading import save_pretrained
    from parallel_b200.models.qwen3 import build_model

    tmp = str(tmp_path)
    save_pretrained(build_model(resolve_config("tiny-qwen3"), dtype=torch.float32, seed=0), f"{tmp}/init")
    full = _run_dist(tmp, topo + [f"config.checkpoint_dir={tmp}/ckpt"], port)
    assert sorted(full) == [1, 2, 3, 4], full
    manifest = f"{tmp}/ckpt/step-00000002/manifest.json"
    assert os.path.isfile(manifest)
    resumed = _run_dist(tmp, topo + [f"config.resume_from={tmp}/ckpt/step-00000002",
                                     f"config.checkpoint_dir={tmp}/c2"], port + 1)
    assert sorted(resumed) == [3, 4], resumed
    for s in (3, 4):
        assert resumed[s] == full[s], (full, resumed)


def test_train_cli_real_data_path_with_local_tokenizer_and_parquet(tmp_path):
    """data.synthetic=false end to end: a tokenizer saved next to the model
    (built offline), parquet shards in data.dir (the last one is validation),
    best-fit packed batches, eval in bits per byte, and an exact resume of
    the data stream from a checkpoint."""
    import pyarrow as pa
    import pyarrow.parquet as pq
    from tokenizers import Tokenizer, models, pre_tokenizers, trainers
    from transformers import PreTrainedTokenizerFast

    from parallel_b200.models.config import resolve_config
    from parallel_b200.models.loading import save_pretrained
    from parallel_b200.models.qwen3 import build_model

    tmp = str(tmp_path)
    words = ["alpha", "beta", "gamma", "delta", "epsilon", "zeta", "eta", "theta", "iota", "kappa"]
    g = torch.Generator().manual_seed(0)
    texts = [" ".join(words[int(i)] for i in torch.randint(0, 10, (int(n),), generator=g))
             for n in torch.randint(3, 40, (400,), generator=g)]
    tok = Tokenizer(models.BPE(unk_token="<unk>"))
    tok.pre_tokenizer = pre_tokenizers.ByteLevel(add_prefix_space=False)
    tok.train_from_iterator(texts, trainers.BpeTrainer(vocab_size=300, special_tokens=["<unk>", "<bos>"],
                                                       initial_alphabet=pre_tokenizers.ByteLevel.alphabet()))
    save_pretrained(build_model(resolve_config("tiny-qwen3"), dtype=torch.float32, seed=0), f"{tmp}/init")
    PreTrainedTokenizerFast(tokenizer_object=tok, bos_token="<bos>", unk_token="<unk>").save_pretrained(f"{tmp}/init")
    os.makedirs(f"{tmp}/data")
    for i, part in enumerate((texts[:300], texts[300:])):
        pq.write_table(pa.table({"text": part}), f"{tmp}/data/shard_{i:05d}.parquet", row_group_size=50)
    common = ["data.synthetic=false", f"data.dir={tmp}/data", "config.grad_accum_steps=1",
              "config.eval_interval=2", "config.eval_steps=2"]
    out_full = _run(tmp, common)
    assert sorted(out_full) == [1, 2, 3, 4], out_full
    state = torch.load(f"{tmp}/ckpt/step-00000002/rank-state-00000.pt", weights_only=False)
    dl = state["dataloader"]
    assert "pq_idx" in dl and "doc_buffer" in dl and not dl.get("synthetic"), dl.keys()
    resumed = _run(tmp, common + [f"config.resume_from={tmp}/ckpt/step-00000002", f"config.checkpoint_dir={tmp}/c2"])
    for s in (3, 4):
        assert resumed[s] == out_full[s], (out_full, resumed)


def test_train_cli_torch_profiler_and_collective_lines(tmp_path):
    """engine.torch_profiler writes one gzip trace for the rank after its
    warm-up / active steps; engine.collective_profiling logs [COLLECTIVE] lines
    for every step (2 gloo ranks, FSDP)."""
    from parallel_b200.models.config import resolve_config
    from parallel_b200.models.loading import save_pretrained
    from parallel_b200.models.qwen3 import build_model

    tmp = str(tmp_path)
    save_pretrained(build_model(resolve_config("tiny-qwen3"), dtype=torch.float32, seed=0), f"{tmp}/init")
    env = dict(os.environ, PYTHONPATH=ROOT, WANDB_MODE="disabled")
    args = [sys.executable, "-m", "torch.distributed.run", "--nproc-per-node", "2", "--master-addr", "127.0.0.1",
            "--master-port", "29651", "-m", "parallel_b200.train", f"model.name={tmp}/init",
            "config.device_type=cpu", "config.backend=gloo", "config.use_amp=false", "data.synthetic=true",
            "config.max_steps=3", "config.eval_interval=100", "config.eval_steps=1", "parallel.dp_shard=2",
            "config.checkpoint_interval=0", "model.per_device_batch_size=2", "model.max_seq_length=32",
            "engine.torch_profiler=true", f"engine.torch_profiler_trace_dir={tmp}/traces",
            "engine.torch_profiler_warmup_steps=1", "engine.torch_profiler_active_steps=1",
            "engine.collective_profiling=true"]
    out = subprocess.run(args, env=env, cwd=tmp, capture_output=True, text=True, timeout=300)
    assert out.returncode == 0, out.stderr[-3000:]
    text = out.stdout + out.stderr
    traces = sorted(os.listdir(f"{tmp}/traces"))
    assert [t for t in traces if t.startswith("rank0")] and [t for t in traces if t.startswith("rank1")], traces
    lines = [l for l in text.splitlines() if "[COLLECTIVE]" in l]
    assert any("fsdp_all_gather" in l for l in lines) and any("fsdp_reduce_scatter" in l for l in lines), lines[:5]
