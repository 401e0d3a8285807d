"""YAML + dot-list configuration loader."""
import textwrap

from parallel_b200.config import Config, from_dotlist, load_cfg, merge, parse_scalar


def test_defaults_match_reference_keys():
    c = load_cfg(argv=[])
    for section, keys in {
        "model": ["name", "max_seq_length", "per_device_batch_size", "learning_rate", "clip_grad_norm",
                  "output_router_logits"],
        "optim": ["adam_beta1", "adam_beta2", "weight_decay"],
        "config": ["device_type", "backend", "use_amp", "amp_dtype", "grad_accum_steps", "max_steps",
                   "eval_interval", "eval_steps", "checkpoint_interval", "checkpoint_dir", "resume_from"],
        "engine": ["cpu_offload", "activation_checkpoint", "checkpoint_every_n", "find_unused_parameters",
                   "overlap_backward_reductions", "collective_profiling", "torch_profiler",
                   "torch_profiler_trace_dir", "torch_profiler_warmup_steps", "torch_profiler_active_steps",
                   "compile"],
        "data": ["dir"],
        "parallel": ["dp_replicate", "dp_shard", "tp", "cp", "sp", "ep", "expert_tp", "pp"],
    }.items():
        for k in keys:
            assert k in c[section], (section, k)
    assert c.model.learning_rate == 1e-5 and isinstance(c.model.learning_rate, float)
    assert c.config.resume_from is None
    assert c.get("seed", 42) == 42


def test_yaml_then_dotlist_override_order(tmp_path):
    y = tmp_path / "o.yaml"
    y.write_text(textwrap.dedent("""
        parallel:
          tp: 2
          sp: 2
        model:
          learning_rate: 3e-4
    """))
    c = load_cfg(argv=[str(y), "parallel.tp=4", "engine.activation_checkpoint=true", "new.key=hello"])
    assert c.parallel.tp == 4 and c.parallel.sp == 2
    assert c.model.learning_rate == 3e-4
    assert c.engine.activation_checkpoint is True
    assert c.new.key == "hello"
    assert c.parallel.dp_shard == 1


def test_scalars_and_merge():
    assert parse_scalar("1e-5") == 1e-5 and parse_scalar("7") == 7 and parse_scalar("null") is None
    assert parse_scalar("false") is False and parse_scalar("abc") == "abc"
    m = merge(Config({"a": {"b": 1, "c": 2}}), from_dotlist(["a.c=3", "a.d.e=4"]))
    assert m.to_container() == {"a": {"b": 1, "c": 3, "d": {"e": 4}}}
