"""Worker of tests/test_multigpu_oracle.py, launched with torchrun (one process
per GPU): trains a small Qwen3 / Qwen3-MoE for two AdamW steps with the
parallel layout named by PB_ORACLE_CASE on the GPUs' default (NVLink /
fused) data plane, saves an exact-topology checkpoint, restores it into a
fresh engine, and continues both engines for one more step.  Rank 0 writes
the losses, gradient norms and portable states for the test to compare with
a single-process fp32 run of the same model and data."""
import os
import sys
from datetime import timedelta

import torch
import torch.distributed as dist

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))

CASES = {
    # case: (model preset, parallel sizes as a function of the world size)
    "fsdp": ("small-qwen3", lambda w: {"dp_shard": w}),
    "dp_replicate": ("small-qwen3", lambda w: {"dp_replicate": w}),
    "hsdp": ("small-qwen3", lambda w: {"dp_replicate": 2, "dp_shard": w // 2}),
    "tp_sp": ("small-qwen3", lambda w: {"tp": w, "sp": w}),
    "moe_tp_ep_sp_fsdp": ("small-qwen3-moe", lambda w: {"tp": 2, "sp": 2, "ep": 2, "dp_shard": w // 2}),
}
B, S, STEPS = 2, 512, 2


def data(world, dp):
    g = torch.Generator().manual_seed(1234)
    return [torch.randint(0, 2048, (B * dp, S + 1), generator=g) for _ in range(STEPS)]


def build_engine(cfg, pc):
    from parallel_b200.models.loading import load_causal_lm
    from parallel_b200.parallel.engine import ParallelEngine

    model, plan = load_causal_lm(cfg, pc, dtype=torch.bfloat16)
    if plan is not None or pc.dp_shard_size <= 1:  # FSDP places its own shards
        model.to(pc.device)
    return ParallelEngine(model, None, pc, cfg, pc.device, mp_plan=plan)


def graph_vs_eager(cfg, pc, tmp, rank):
    """The whole-step CUDA graph (engine.compile's path: one eager step on the
    capture stream, then capture and replay) against eager steps on the same
    four batches."""
    g = torch.Generator().manual_seed(77)
    batches = [torch.randint(0, 2048, (B * pc.data_world_size, S + 1), generator=g) for _ in range(4)]
    runs = {}
    for mode in ("eager", "graph"):
        eng = build_engine(cfg, pc)
        if mode == "graph":
            eng.enable_graph_capture(warmup_steps=1)
        losses = []
        for tok in batches:
            mine = tok[pc.data_rank * B:(pc.data_rank + 1) * B].cuda()
            loss = eng.train_step(mine[:, :-1], mine[:, 1:])
            losses.append(float(eng.reduce_loss(loss)))
        runs[mode] = (losses, eng.state_dict(), eng._graph is not None)
        eng.release_graph()
    if rank == 0:
        torch.save(runs, os.path.join(tmp, "graph_result.pt"))
    dist.barrier()
    dist.destroy_process_group()


def main():
    from parallel_b200.config import from_dotlist, load_cfg, merge
    from parallel_b200.ops._ext import check_device_errors
    from parallel_b200.state import ParallelConfig

    local = int(os.environ["LOCAL_RANK"])
    torch.cuda.set_device(local)
    dist.init_process_group("nccl", timeout=timedelta(seconds=180), device_id=torch.device("cuda", local))
    world, rank = dist.get_world_size(), dist.get_rank()
    case = os.environ["PB_ORACLE_CASE"]
    tmp = os.environ["PB_ORACLE_TMP"]
    name, layout = CASES[case]
    par = layout(world)
    path = os.path.join(tmp, "model")
    over = [f"model.name={path}", "config.device_type=cuda", "config.backend=nccl", "model.learning_rate=1e-3",
            "model.clip_grad_norm=1.0", "optim.weight_decay=0.01", "engine.activation_checkpoint=true",
            f"engine.overlap_backward_reductions={os.environ.get('PB_ORACLE_OVERLAP', 'true')}"]
    over += [f"parallel.{k}={v}" for k, v in par.items()]
    cfg = merge(load_cfg(argv=[]), from_dotlist(over))
    pc = ParallelConfig(cfg)
    pc.set_device_mesh("cuda")
    dp = pc.data_world_size
    batches = data(world, dp)
    if os.environ.get("PB_ORACLE_GRAPH") == "1":
        return graph_vs_eager(cfg, pc, tmp, rank)
    eng = build_engine(cfg, pc)
    losses, norms = [], []
    for tok in batches:
        mine = tok[pc.data_rank * B:(pc.data_rank + 1) * B].cuda()
        loss = eng.forward(mine[:, :-1], mine[:, 1:]).loss
        eng.backward(loss)
        eng.step()
        norms.append(float(eng.last_grad_norm))
        losses.append(float(eng.reduce_loss(loss)))
    state = eng.state_dict()
    ck = os.path.join(tmp, "ckpt")
    eng.save_checkpoint(ck, step=STEPS)
    eng2 = build_engine(cfg, pc)
    eng2.load_checkpoint(ck)
    cont = []
    for e in (eng, eng2):
        mine = batches[0][pc.data_rank * B:(pc.data_rank + 1) * B].cuda()
        loss = e.forward(mine[:, :-1], mine[:, 1:]).loss
        e.backward(loss)
        e.step()
        cont.append(float(e.reduce_loss(loss)))
    after = [eng.state_dict(), eng2.state_dict()]
    torch.cuda.synchronize()
    check_device_errors()
    for e in (eng, eng2):
        e.release_graph()
    if rank == 0:
        torch.save({"losses": losses, "norms": norms, "state": state, "cont": cont, "after": after, "par": par,
                    "dp": dp}, os.path.join(tmp, "result.pt"))
    dist.barrier()
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
