"""Worker launched by tests/test_multigpu.py with torchrun (one process per GPU)."""
import json
import os
import sys
from datetime import timedelta

import torch
import torch.distributed as dist

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))


def run_engine(collectives, data, layers=2):
    from parallel_b200.config import from_dotlist, load_cfg, merge
    from parallel_b200.models.config import resolve_config
    from parallel_b200.models.qwen3 import build_model
    from parallel_b200.parallel.engine import ParallelEngine
    from parallel_b200.state import ParallelConfig

    world = dist.get_world_size()
    cfg = merge(load_cfg(argv=[]), from_dotlist([
        "config.device_type=cuda", "model.learning_rate=1e-3", f"parallel.dp_shard={world}",
        "engine.activation_checkpoint=true", f"engine.collectives={collectives}"]))
    pc = ParallelConfig(cfg)
    pc.set_device_mesh("cuda")
    mcfg = resolve_config("Qwen/Qwen3-0.6B", num_hidden_layers=layers, vocab_size=4096)
    m = build_model(mcfg, dtype=torch.bfloat16, seed=0)
    eng = ParallelEngine(m, None, pc, cfg, pc.device)
    losses = []
    r = dist.get_rank()
    for tok in data:
        b = tok.shape[0] // world
        mine = tok[r * b:(r + 1) * b].cuda()
        loss = eng.forward(mine[:, :-1], mine[:, 1:]).loss
        eng.backward(loss)
        eng.step()
        losses.append(eng.reduce_loss(loss).item())
    state = eng.state_dict()
    from parallel_b200.ops._ext import check_device_errors

    torch.cuda.synchronize()
    check_device_errors()
    return losses, state, eng.fsdp_wrapper.coll.name


def run_sp(collectives, data, steps_grads, moe=False, sp=True):
    """Qwen3 (head_dim 128) with tp = sp = world: the fused NVLink sequence-parallel
    kernels (collectives != nccl) against the NCCL path.  Returns losses and
    the local gradient shards after one backward."""
    from parallel_b200.config import from_dotlist, load_cfg, merge
    from parallel_b200.models.config import resolve_config
    from parallel_b200.models.qwen3 import build_model
    from parallel_b200.parallel.engine import ParallelEngine
    from parallel_b200.state import ParallelConfig

    from parallel_b200.models.loading import load_causal_lm, save_pretrained

    world = dist.get_world_size()
    path = os.path.join(os.environ.get("PB_TEST_TMP", "/tmp"), "sp_ckpt")
    if dist.get_rank() == 0:
        if moe:
            mcfg = resolve_config("small-qwen3-moe", num_hidden_layers=2, vocab_size=2048)
        else:
            mcfg = resolve_config("small-qwen3", num_hidden_layers=2, vocab_size=2048, hidden_size=512,
                                  intermediate_size=1024)
        model = build_model(mcfg, dtype=torch.bfloat16, seed=0)
        if moe:
            # spread the router logits so that the two paths' different (but
            # both valid) rounding of the expert combine cannot flip a near-tie
            # top-k choice in the next layer: both then route identically
            with torch.no_grad():
                for n, p in model.named_parameters():
                    if n.endswith("mlp.gate.weight"):
                        p.mul_(30.0)
        save_pretrained(model, path)
    dist.barrier()
    par = [f"parallel.tp={world}"] + ([f"parallel.sp={world}"] if sp else []) + \
        ([f"parallel.ep={world}"] if moe else [])
    cfg = merge(load_cfg(argv=[]), from_dotlist([
        "config.device_type=cuda", "model.learning_rate=1e-3", f"model.name={path}",
        "engine.activation_checkpoint=false", f"engine.collectives={collectives}"] + par))
    pc = ParallelConfig(cfg)
    pc.set_device_mesh("cuda")
    m, plan = load_causal_lm(cfg, pc, dtype=torch.bfloat16)
    m.to(pc.device)
    eng = ParallelEngine(m, None, pc, cfg, pc.device, mp_plan=plan)
    ctx0 = eng.model.model.layers[0]._ctx
    if moe and sp:
        fused = type(ctx0.expert_runtime.transport).__name__ == "PeerExpertTransport"
    elif moe:
        fused = getattr(ctx0.expert_runtime, "fused", None) is not None
    else:
        fused = ctx0.fused_tp is not None
    losses, grads = [], {}
    for i, tok in enumerate(data):
        tok = tok.cuda()
        loss = eng.forward(tok[:, :-1], tok[:, 1:]).loss
        eng.backward(loss)
        if i == 0:
            for n, p in eng.model.named_parameters():
                if p.grad is not None:
                    grads[n] = p.grad.detach().float().cpu()
        eng.step()
        losses.append(eng.reduce_loss(loss).item())
    from parallel_b200.ops._ext import check_device_errors

    torch.cuda.synchronize()
    check_device_errors()
    return losses, grads, fused


def main_sp():
    local = int(os.environ["LOCAL_RANK"])
    torch.cuda.set_device(local)
    dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=torch.device("cuda", local))
    world = dist.get_world_size()
    g = torch.Generator().manual_seed(0)
    data = [torch.randint(0, 2048, (2, 256 * world + 1), generator=g) for _ in range(3)]
    moe = os.environ.get("PB_TEST_MOE") == "1"
    sp = os.environ.get("PB_TEST_SP", "1") == "1"
    l_f, g_f, fused = run_sp("p2p", data, 1, moe, sp)
    l_n, g_n, fused_n = run_sp("nccl", data, 1, moe, sp)
    worst = (0.0, "")
    for k in g_n:
        a, b = g_f[k], g_n[k]
        worst = max(worst, (((a - b).norm() / (b.norm() + 1e-12)).item(), k))
    every = [None] * dist.get_world_size()
    dist.all_gather_object(every, worst)
    worst = max(every)
    if dist.get_rank() == 0:
        with open(os.environ["PB_TEST_OUT"], "w") as f:
            json.dump({"fused": l_f, "nccl": l_n, "used_fused": [fused, fused_n], "grad_rel_diff": worst[0],
                       "worst_param": worst[1]}, f)
    dist.barrier()
    dist.destroy_process_group()


def main_small():
    """P2P small all-reduce (sum / max / log-sum-exp merge) against NCCL, over
    varying sizes (both slot parities) and inside a replayed CUDA graph."""
    from parallel_b200.ops._ext import check_device_errors
    from parallel_b200.parallel.comm.p2p import P2PSmallAllReduce

    local = int(os.environ["LOCAL_RANK"])
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=dev)
    rank = dist.get_rank()
    group = dist.group.WORLD
    ar = P2PSmallAllReduce.get(group, dev)
    worst = 0.0
    g = torch.Generator(device="cpu").manual_seed(100 + rank)
    for n in (1, 2, 1000, 37, 40000, 5, 16384 * 3):
        x = torch.randn(n, generator=g).to(dev)
        for op, red in (("sum", dist.ReduceOp.SUM), ("max", dist.ReduceOp.MAX)):
            ref = x.clone()
            dist.all_reduce(ref, op=red)
            got = ar.all_reduce_(x.clone(), op)
            worst = max(worst, ((got - ref).abs().max() / (ref.abs().max() + 1e-12)).item())
    for rows in (7, 2048, 8192):
        m = torch.randn(rows, generator=g).to(dev) * 4
        se = torch.rand(rows, generator=g).to(dev) + 0.5
        tg = torch.randn(rows, generator=g).to(dev)
        lse, tsum = ar.lse_merge(m, se, tg)
        gm = m.clone()
        dist.all_reduce(gm, op=dist.ReduceOp.MAX)
        gs = se * torch.exp(m - gm)
        dist.all_reduce(gs)
        ref_lse = gm + torch.log(gs)
        ref_t = tg.clone()
        dist.all_reduce(ref_t)
        worst = max(worst, ((lse - ref_lse).abs().max() / ref_lse.abs().max()).item(),
                    ((tsum - ref_t).abs().max() / ref_t.abs().max()).item())
    # graph replay: the epochs live on the device
    x = torch.ones(300, device=dev) * (rank + 1)
    y = torch.empty_like(x)
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        y.copy_(x)
        ar.all_reduce_(y, "sum")
    torch.cuda.current_stream().wait_stream(s)
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=s):
        y.copy_(x)
        ar.all_reduce_(y, "sum")
        ar.all_reduce_(y, "sum")
    W = dist.get_world_size()
    for i in range(3):
        x.fill_(rank + 1 + i)
        graph.replay()
        torch.cuda.synchronize()
        expect = W * sum(r + 1 + i for r in range(W))
        worst = max(worst, abs(float(y[0]) - expect) / expect)
    graph.reset()
    check_device_errors()
    t = torch.tensor([worst], device=dev)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    if rank == 0:
        with open(os.environ["PB_TEST_OUT"], "w") as f:
            json.dump({"worst": t.item()}, f)
    dist.barrier()
    dist.destroy_process_group()


def main_nvls():
    """In-switch all-reduce (multimem) against an fp32 sum of the same bf16
    inputs: several tensors, a mean scale, the replicate-mean wrapper and a
    replayed CUDA graph.  Writes {"skipped": why} where the fabric has no NVLS."""
    from parallel_b200.ops._ext import check_device_errors
    from parallel_b200.parallel.comm.p2p import NvlsAllReduce, ReplicaMeanAllReduce

    local = int(os.environ["LOCAL_RANK"])
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=dev)
    rank, W = dist.get_rank(), dist.get_world_size()
    group = dist.group.WORLD
    out = {}
    nv = NvlsAllReduce.get(group, dev, 1 << 22, force=True)
    if nv is None:
        out["skipped"] = "no switch multicast on this fabric (probe or multicast address)"
    else:
        g = torch.Generator(device="cpu").manual_seed(7 + rank)
        worst = 0.0
        for sizes, scale in (([8], 1.0), ([4096, 1 << 20, 24], 1.0), ([3 * (1 << 20)], 1.0 / W)):
            xs = [torch.randn(n, generator=g).to(dev, torch.bfloat16) for n in sizes]
            ref = [x.float() for x in xs]
            for r in ref:
                dist.all_reduce(r)
            got = [x.clone() for x in xs]
            nv.all_reduce_(got, scale)
            for a, b in zip(got, ref):
                b = (b * scale).to(torch.bfloat16).float()
                worst = max(worst, ((a.float() - b).abs().max() / (b.abs().max() + 1e-12)).item())
        # the replicate mean takes the NVLS path when PB_NVLS=1
        grads = [torch.randn(n, generator=g).to(dev, torch.bfloat16) for n in (1024, 65536)]
        ref = [t.float() for t in grads]
        for r in ref:
            dist.all_reduce(r)
        rm = ReplicaMeanAllReduce.get(group, dev, grads)
        out["replica_uses_nvls"] = rm is not None and rm.nvls is not None
        rm.mean_(grads)
        for a, b in zip(grads, ref):
            b = (b / W).to(torch.bfloat16).float()
            worst = max(worst, ((a.float() - b).abs().max() / (b.abs().max() + 1e-12)).item())
        # graph replay (device epochs in the barriers)
        x = torch.full((4096,), float(rank + 1), device=dev, dtype=torch.bfloat16)
        y = torch.empty_like(x)
        s = torch.cuda.Stream()
        s.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(s):
            nv.all_reduce_([x], 1.0, outs=[y])
        torch.cuda.current_stream().wait_stream(s)
        torch.cuda.synchronize()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=s):
            nv.all_reduce_([x], 1.0, outs=[y])
        for i in range(3):
            x.fill_(float(rank + 1 + i))
            graph.replay()
            torch.cuda.synchronize()
            expect = sum(r + 1 + i for r in range(W))
            worst = max(worst, abs(float(y[0]) - expect) / expect, abs(float(y[-1]) - expect) / expect)
        graph.reset()
        check_device_errors()
        out["worst"] = worst
    t = torch.tensor([out.get("worst", 0.0)], device=dev)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    out["worst"] = t.item()
    if rank == 0:
        with open(os.environ["PB_TEST_OUT"], "w") as f:
            json.dump(out, f)
    dist.barrier()
    dist.destroy_process_group()


def main():
    if os.environ.get("PB_TEST_MODE") == "nvls":
        return main_nvls()
    if os.environ.get("PB_TEST_MODE") == "sp":
        return main_sp()
    if os.environ.get("PB_TEST_MODE") == "small":
        return main_small()
    local = int(os.environ["LOCAL_RANK"])
    torch.cuda.set_device(local)
    dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=torch.device("cuda", local))
    world = dist.get_world_size()
    g = torch.Generator().manual_seed(0)
    data = [torch.randint(0, 4096, (2 * world, 257), generator=g) for _ in range(3)]
    l_p2p, s_p2p, n1 = run_engine("p2p", data)
    l_nccl, s_nccl, n2 = run_engine("nccl", data)
    out = {"p2p": l_p2p, "nccl": l_nccl, "names": [n1, n2]}
    if dist.get_rank() == 0:
        worst = 0.0
        for k in s_p2p:
            a, b = s_p2p[k].float(), s_nccl[k].float()
            worst = max(worst, ((a - b).norm() / (b.norm() + 1e-12)).item())
        out["state_rel_diff"] = worst
        with open(os.environ["PB_TEST_OUT"], "w") as f:
            json.dump(out, f)
    dist.barrier()
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
