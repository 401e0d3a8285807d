"""Fused-collective micro-benchmarks: this repository's NVLink kernels against
the reference's composition (NCCL collective + cuBLAS GEMM), one process per GPU.

    torchrun --nproc-per-node N --master-addr 127.0.0.1 -m parallel_b200.parallel.collective_bench \
        [--cases ag_gemm,gemm_rs,fsdp_ag,fsdp_rs,ep,ce] [--quick] [--iters 10]

Cases (bf16 N(0,1) inputs from a fixed seed):

* ``ag_gemm``  all-gather of the sequence shard -> column-parallel GEMM
  (``FusedSequenceParallel.all_gather_gemm`` vs ``all_gather_into_tensor`` + ``torch.matmul``;
  ``pull_us``: the same in pull mode, peer gather kernel then plain GEMM);
* ``gemm_rs``  row-parallel GEMM -> reduce-scatter (``gemm_reduce_scatter`` vs
  ``torch.matmul`` + ``reduce_scatter_tensor``; ``pull_us``: GEMM into the local
  symmetric buffer, then each owner pulls and sums its rows);
* ``fsdp_ag`` / ``fsdp_rs``  flat-buffer all-gather / reduce-scatter (peer gather / N-peer
  reduce kernels vs NCCL);
* ``ep``  one MoE layer forward + backward, top-8 routes over 128 experts: the
  device-resident peer-memory path (routing plan, dispatch into the owners' padded
  expert matrices, grouped tcgen05 GEMMs, weighted pull-combine) vs NCCL variable
  all-to-alls with host-read splits around ``torch._grouped_mm``; uniform and skewed
  routing;
* ``ce``  vocabulary-parallel LM head + cross-entropy (peer log-sum-exp merge vs NCCL
  all-reduces);
* ``all_reduce``  flat bf16 all-reduce: in-switch NVLS (``multimem``) where the
  fabric has it, the peer-load path as ``pull_us``, NCCL as the baseline (not in
  the default list: ``--cases all_reduce``).

Every time is device time with CUDA events after warm-up, the max over ranks.
``roofline`` is the slower of the FLOPs at the measured bf16 GEMM peak and the
bytes each GPU must receive over NVLink at the measured 770 GB/s peer copy;
``frac`` = roofline / achieved time.  Rank 0 prints one JSON line per case.
"""
from __future__ import annotations

import argparse
import json
import os
from datetime import timedelta

import torch
import torch.distributed as dist



def _measured_gemm_peak(default: float = 1.646e15) -> float:
    """The cuBLAS bf16 burst peak measured on the machine (``MEASURED_PEAKS.json``
    beside the repository, ``bf16_tflops``), else the last measurement on a
    B200 of this pool."""
    path = os.path.join(os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__)))),
                        "MEASURED_PEAKS.json")
    try:
        return float(json.load(open(path))["bf16_tflops"]) * 1e12
    except Exception:
        return default


GEMM_PEAK = _measured_gemm_peak()  # FLOP/s
LINK_BW = 770e9       # measured peer copy per direction (B/s)


def _time(fn, warmup, iters):
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    dist.barrier()
    torch.cuda.synchronize()
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record()
    for _ in range(iters):
        fn()
    e.record()
    torch.cuda.synchronize()
    t = torch.tensor([s.elapsed_time(e) / iters * 1e3], device="cuda")  # us
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t)


def _report(case, shape, ours_us, base_us, flops, link_bytes, pull_us=None):
    roof = max(flops / GEMM_PEAK, link_bytes / LINK_BW) * 1e6
    out = {"case": case, "shape": shape, "ours_us": round(ours_us, 1), "nccl_cublas_us": round(base_us, 1),
           "speedup": round(base_us / ours_us, 3), "roofline_us": round(roof, 1),
           "frac_of_roofline": round(roof / ours_us, 3)}
    if pull_us is not None:
        # the same operation in pull mode (collective kernel + plain GEMM, no
        # communication inside the GEMM)
        out.update(pull_us=round(pull_us, 1), pull_speedup=round(base_us / pull_us, 3),
                   pull_frac_of_roofline=round(roof / pull_us, 3))
    return out


def case_ag_gemm(W, rank, dev, M, K, N, warmup, iters):
    from .model_parallel.fused_sp import FusedSequenceParallel

    g = torch.Generator(device="cpu").manual_seed(rank)
    x = torch.randn(M // W, K, generator=g).to(dev, torch.bfloat16)
    w = (torch.randn(N, K, generator=g) / K ** 0.5).to(dev, torch.bfloat16)
    sp = FusedSequenceParallel(dist.group.WORLD, dev)
    if not sp.supports(1, M, K):
        return None
    ours = _time(lambda: sp.all_gather_gemm(x, w, 1, M), warmup, iters)
    pull = FusedSequenceParallel(dist.group.WORLD, dev, mode="pull")
    t_pull = _time(lambda: pull.all_gather_gemm(x, w, 1, M), warmup, iters)
    full = torch.empty(M, K, device=dev, dtype=torch.bfloat16)

    def base():
        dist.all_gather_into_tensor(full, x)
        torch.matmul(full, w.t())

    return _report("ag_gemm", [M, K, N], ours, _time(base, warmup, iters), 2 * M * K * N, (W - 1) * (M // W) * K * 2,
                   t_pull)


def case_gemm_rs(W, rank, dev, M, K, N, warmup, iters):
    from .model_parallel.fused_sp import FusedSequenceParallel

    g = torch.Generator(device="cpu").manual_seed(rank)
    a = torch.randn(M, K, generator=g).to(dev, torch.bfloat16)
    w = (torch.randn(N, K, generator=g) / K ** 0.5).to(dev, torch.bfloat16)
    sp = FusedSequenceParallel(dist.group.WORLD, dev)
    if not sp.supports(1, M, N):
        return None
    ours = _time(lambda: sp.gemm_reduce_scatter(a, w, 1, M), warmup, iters)
    pull = FusedSequenceParallel(dist.group.WORLD, dev, mode="pull")
    t_pull = _time(lambda: pull.gemm_reduce_scatter(a, w, 1, M), warmup, iters)
    out = torch.empty(M // W, N, device=dev, dtype=torch.bfloat16)

    def base():
        dist.reduce_scatter_tensor(out, torch.matmul(a, w.t()))

    return _report("gemm_rs", [M, K, N], ours, _time(base, warmup, iters), 2 * M * K * N, (W - 1) * (M // W) * N * 2,
                   t_pull)


def _flat_buffers(W, dev, nbytes):
    from .comm.p2p import SymmBuffer

    n = nbytes // 2 // (8 * W) * (8 * W)
    buf = SymmBuffer(n, torch.bfloat16, dev, dist.group.WORLD)
    buf.tensor[:n].normal_()
    return buf, n


def case_fsdp_ag(W, rank, dev, nbytes, warmup, iters):
    from ..ops._ext import ext

    buf, n = _flat_buffers(W, dev, nbytes)
    shard = n // W
    full = torch.empty(n, device=dev, dtype=torch.bfloat16)
    order = [(rank + i) % W for i in range(W)]  # as the FSDP gather: own shard first, then rank+1, ...
    src = [buf.peer_ptrs[r] for r in order]
    dst = [full.data_ptr() + r * shard * 2 for r in order]

    def ours():
        buf.barrier(0, 60.0)
        ext().p2p_copy(src, dst, [shard * 2] * W)

    local = buf.tensor[:shard]
    t_ours = _time(ours, warmup, iters)
    t_base = _time(lambda: dist.all_gather_into_tensor(full, local), warmup, iters)
    return _report("fsdp_ag", [n * 2 // (1 << 20), "MB"], t_ours, t_base, 0, (W - 1) * shard * 2)


def case_fsdp_rs(W, rank, dev, nbytes, warmup, iters):
    from ..ops._ext import ext

    buf, n = _flat_buffers(W, dev, nbytes)
    shard = n // W
    out = torch.empty(shard, device=dev, dtype=torch.bfloat16)
    src = [[p + rank * shard * 2] for p in buf.peer_ptrs]

    def ours():
        buf.barrier(1, 60.0)
        ext().p2p_reduce(src, [out.data_ptr()], [shard], 1.0 / W, False)

    t_ours = _time(ours, warmup, iters)
    full = buf.tensor[:n]
    t_base = _time(lambda: dist.reduce_scatter_tensor(out, full), warmup, iters)
    return _report("fsdp_rs", [n * 2 // (1 << 20), "MB"], t_ours, t_base, 0, (W - 1) * shard * 2)


def case_all_reduce(W, rank, dev, nbytes, warmup, iters):
    """bf16 SUM all-reduce of one flat buffer.  ours: the in-switch NVLS
    all-reduce (``NvlsAllReduce``: multimem.ld_reduce of this rank's slice,
    multimem.st of the sum) when the fabric has it, else the peer-load mean
    path; pull: the peer-load path (copy into a symmetric slot, barrier, every
    rank reads and sums all slots); baseline: NCCL all_reduce.  Roofline: the
    bytes each GPU receives, S (1 + 1/W) in the switch scheme (its reduced
    slice, then every slice of the broadcast), 2 S (W - 1) / W otherwise."""
    from .comm.p2p import NvlsAllReduce, ReplicaMeanAllReduce

    n = nbytes // 2
    x = torch.randn(n, generator=torch.Generator().manual_seed(rank)).to(dev, torch.bfloat16)
    y = torch.empty_like(x)
    nv = NvlsAllReduce.get(dist.group.WORLD, dev, n, force=True)
    prev = os.environ.get("PB_NVLS")
    os.environ["PB_NVLS"] = "0"
    try:
        peer = ReplicaMeanAllReduce.get(dist.group.WORLD, dev, [y])
    finally:
        if prev is None:
            os.environ.pop("PB_NVLS", None)
        else:
            os.environ["PB_NVLS"] = prev
    t_pull = _time(lambda: peer.mean_([y]), warmup, iters)
    t_ours = _time(lambda: nv.all_reduce_([x], 1.0, outs=[y]), warmup, iters) if nv is not None else t_pull
    t_base = _time(lambda: dist.all_reduce(y), warmup, iters)
    out = _report("all_reduce" + ("_nvls" if nv is not None else "_p2p"), [nbytes >> 20, "MB"], t_ours, t_base, 0,
                  nbytes * (W + 1) / W if nv is not None else 2 * nbytes * (W - 1) / W, pull_us=t_pull)
    if nv is not None:
        # numerics of the timed path: against an fp32 NCCL sum of the same bf16 inputs
        ref = x.float()
        dist.all_reduce(ref)
        nv.all_reduce_([x], 1.0, outs=[y])
        err = ((y.float() - ref).abs().max() / ref.abs().max().clamp_min(1e-12)).reshape(1)
        dist.all_reduce(err, op=dist.ReduceOp.MAX)
        out["max_rel_err"] = float(err)
    return out


def _torch_experts(x, idx, w, w_gu, w_d):
    """Reference-style expert MLPs of locally received routes: sort by expert,
    torch grouped GEMMs (``torch._grouped_mm``, the op HF's grouped expert path
    calls), SwiGLU, routing-weight scaling, unsort."""
    import torch.nn.functional as F

    flat = idx.reshape(-1)
    order = torch.argsort(flat, stable=True)
    counts = torch.bincount(flat, minlength=w_gu.shape[0])
    offs = torch.cumsum(counts, 0).to(torch.int32)
    xs = x.index_select(0, order)
    gu = torch._grouped_mm(xs, w_gu.transpose(1, 2), offs=offs)
    g, u = gu.chunk(2, dim=-1)
    y = torch._grouped_mm((F.silu(g) * u).contiguous(), w_d.transpose(1, 2), offs=offs)
    y = y * w.reshape(-1)[order, None].to(y.dtype)
    return torch.empty_like(y).index_copy_(0, order, y)


def case_ep(W, rank, dev, tokens, hidden, experts, top_k, warmup, iters, inter=768, skew=0.0):
    """One MoE layer forward + backward: route exchange, expert MLPs, combine.
    Ours: the device-resident peer-memory path (``PeerExpertTransport``);
    baseline: NCCL variable all-to-alls with host-read splits around torch
    grouped GEMMs (the reference's composition)."""
    from ..ops.moe import routed_experts
    from .model_parallel.expert_parallel import ExpertPartition
    from .model_parallel.p2p_dispatch import PeerExpertTransport
    from .model_parallel.token_dispatch import TokenDispatcher

    g = torch.Generator(device="cpu").manual_seed(rank)
    x = torch.randn(tokens, hidden, generator=g).to(dev, torch.bfloat16).requires_grad_(True)
    bias = torch.randn(experts, generator=torch.Generator().manual_seed(7)) * skew
    logits = torch.randn(tokens, experts, generator=g) + bias
    sc, idx = torch.softmax(logits, -1).topk(top_k, -1)
    sc, idx = sc.to(dev).requires_grad_(True), idx.to(dev)
    part = ExpertPartition(experts, W, rank)
    wg = torch.Generator().manual_seed(100 + rank)
    w_gu = (torch.randn(part.local_count, 2 * inter, hidden, generator=wg) * 0.02).to(dev, torch.bfloat16)
    w_d = (torch.randn(part.local_count, hidden, inter, generator=wg) * 0.02).to(dev, torch.bfloat16)
    w_gu.requires_grad_(True)
    w_d.requires_grad_(True)
    transport = PeerExpertTransport(part, dist.group.WORLD, dev)
    nccl = TokenDispatcher(part, dist.group.WORLD)
    dout = torch.randn(tokens, hidden, generator=g).to(dev, torch.bfloat16)

    def ours():
        routed_experts(x, sc, idx, w_gu, w_d, transport).backward(dout)

    def base():
        h, e, s, st = nccl.dispatch(x, idx, sc)
        nccl.combine(_torch_experts(h, e, s, w_gu, w_d), st).backward(dout)

    t_ours = _time(ours, warmup, iters)
    t_base = _time(base, warmup, iters)
    # each route's row crosses the link to its owner and back, forward and backward
    link = 4 * tokens * top_k * hidden * 2 * (W - 1) / W
    flops = 3 * 2 * tokens * top_k * hidden * 3 * inter  # three products, forward + two backward
    return _report("ep_moe_layer" + ("_skew" if skew else ""), [tokens, hidden, experts, top_k], t_ours, t_base,
                   flops, link)


def case_ce(W, rank, dev, tokens, hidden, vocab, warmup, iters):
    from .model_parallel.loss_parallel import vocab_parallel_lm_head_ce

    g = torch.Generator(device="cpu").manual_seed(0)
    h = torch.randn(tokens, hidden, generator=g).to(dev, torch.bfloat16)
    w = (torch.randn(vocab // W, hidden, generator=torch.Generator().manual_seed(rank)) * 0.02).to(dev, torch.bfloat16)
    labels = torch.randint(0, vocab, (tokens,), generator=g).to(dev)
    v0 = rank * (vocab // W)
    grp = dist.group.WORLD
    t_ours = _time(lambda: vocab_parallel_lm_head_ce(h, w, labels, grp, v0, collectives="p2p"), warmup, iters)
    t_base = _time(lambda: vocab_parallel_lm_head_ce(h, w, labels, grp, v0, collectives="nccl"), warmup, iters)
    flops = 3 * 2 * tokens * hidden * (vocab // W)  # logits, dh, dW
    return _report("vocab_parallel_ce", [tokens, hidden, vocab], t_ours, t_base, flops, 3 * tokens * 4 * (W - 1))


def main(argv=None):
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--cases", default="ag_gemm,gemm_rs,fsdp_ag,fsdp_rs,ep,ce")
    ap.add_argument("--quick", action="store_true", help="one shape per case")
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--iters", type=int, default=10)
    args = ap.parse_args(argv)
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=dev)
    W, rank = dist.get_world_size(), dist.get_rank()
    cases = args.cases.split(",")
    gemm_shapes = [(8192, 4096, 4096)] if args.quick else [(4096, 4096, 4096), (16384, 4096, 4096),
                                                          (32768, 4096, 4096), (16384, 4096, 12288)]
    flat = [64 << 20] if args.quick else [8 << 20, 64 << 20, 512 << 20]
    results = []
    for M, K, N in gemm_shapes:
        if "ag_gemm" in cases:
            results.append(case_ag_gemm(W, rank, dev, M, K, N, args.warmup, args.iters))
        if "gemm_rs" in cases:
            results.append(case_gemm_rs(W, rank, dev, M, K, N, args.warmup, args.iters))
    for nb in flat:
        if "fsdp_ag" in cases:
            results.append(case_fsdp_ag(W, rank, dev, nb, args.warmup, args.iters))
        if "fsdp_rs" in cases:
            results.append(case_fsdp_rs(W, rank, dev, nb, args.warmup, args.iters))
    if "all_reduce" in cases:
        for nb in flat:
            results.append(case_all_reduce(W, rank, dev, nb, args.warmup, args.iters))
    if "ep" in cases:
        # tokens per rank (Qwen3-30B-A3B at B=1, S=4096 under sp=4 has 1024), hidden 2048, top-8 of 128
        # experts, expert SwiGLU width 768; uniform routing and an N(0, 2)-biased (skewed) router
        for tokens in ([1024] if args.quick else [1024, 4096]):
            for skew in (0.0, 2.0):
                results.append(case_ep(W, rank, dev, tokens, 2048, 128, 8, args.warmup, args.iters, skew=skew))
    if "ce" in cases:
        results.append(case_ce(W, rank, dev, 16384 if not args.quick else 8192, 1024, 151936, args.warmup,
                               args.iters))
    if rank == 0:
        for r in results:
            if r is not None:
                print(json.dumps(dict(r, n_gpus=W)), flush=True)
    dist.barrier()
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
