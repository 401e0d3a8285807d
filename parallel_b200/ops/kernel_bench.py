"""Micro-benchmarks of the sm_100a kernels at the Qwen3-0.6B training shapes.

    python -m parallel_b200.ops.kernel_bench attn_fwd|attn_bwd|ce|gemm|gemm_vs_cublas|gemm_swiglu|gemm_residual|moe_layer|rmsnorm_bwd|qknorm|qknorm_bwd|wgrad_split|all [--iters N]

Each case runs a few warm-up launches, then times ``--iters`` launches with
CUDA events on the current stream and prints the time per launch and the
achieved TF/s or GB/s.  With ``--iters 1`` and ``--warmup 3`` the same command
is the small case used for profiler captures, after the same command has run
to completion without the profiler:
``ncu --set full --clock-control none -k <kernel> -s 3 -c 1 python -m parallel_b200.ops.kernel_bench <case>
--iters 1 --warmup 3`` (``--clock-control none`` leaves the GPU's clocks alone).
"""
from __future__ import annotations

import argparse
import math

import torch

from ._ext import check_device_errors, ext

B, S, NQ, NKV, D, H, I = 4, 2048, 16, 8, 128, 1024, 3072


def _time(fn, warmup: int, iters: int) -> float:
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record()
    for _ in range(iters):
        fn()
    e.record()
    torch.cuda.synchronize()
    check_device_errors()
    return s.elapsed_time(e) / iters * 1e3  # us


def _attn_inputs():
    T = B * S
    q = torch.randn(T, NQ * D, device="cuda", dtype=torch.bfloat16)
    k = torch.randn(T, NKV * D, device="cuda", dtype=torch.bfloat16)
    v = torch.randn(T, NKV * D, device="cuda", dtype=torch.bfloat16)
    o = torch.empty_like(q)
    lse = torch.zeros(B * NQ * S + 128, device="cuda")
    return q, k, v, o, lse


def case_attn_fwd(warmup, iters):
    C = ext()
    q, k, v, o, lse = _attn_inputs()
    us = _time(lambda: C.attn_fwd(q, k, v, o, lse, B, S, NQ, NKV, 1 / math.sqrt(D), True), warmup, iters)
    flops = 4 * B * NQ * S * S * D / 2
    return f"attention fwd B={B} S={S} heads={NQ}/{NKV} D={D} causal: {us:.1f} us, {flops / us / 1e6:.0f} TF/s"


def case_attn_bwd(warmup, iters):
    C = ext()
    q, k, v, o, lse = _attn_inputs()
    C.attn_fwd(q, k, v, o, lse, B, S, NQ, NKV, 1 / math.sqrt(D), True)
    do = torch.randn_like(q)
    delta = torch.empty(2 * lse.numel(), device="cuda")
    acc = torch.empty(0, device="cuda")
    dq, dk, dv = torch.empty_like(q), torch.empty_like(k), torch.empty_like(v)
    ds = torch.empty(C.attn_bwd_ds_elems(B, S, NQ, True), device="cuda", dtype=torch.bfloat16)
    us = _time(lambda: C.attn_bwd(q, k, v, o, do, lse, delta, acc, dq, dk, dv, B, S, NQ, NKV, 1 / math.sqrt(D), True,
                                  None, ds), warmup, iters)
    flops = 2.5 * 4 * B * NQ * S * S * D / 2
    return f"attention bwd (prep + main + dQ kernels) B={B} S={S} heads={NQ}/{NKV}: {us:.1f} us, {flops / us / 1e6:.0f} TF/s"


def case_gemm(warmup, iters):
    C = ext()
    M, N, K = B * S, (NQ + 2 * NKV) * D, H  # the fused QKV projection
    a = (torch.randn(M, K, device="cuda") * 0.05).to(torch.bfloat16)
    b = (torch.randn(N, K, device="cuda") * 0.05).to(torch.bfloat16)
    out = torch.empty(M, N, device="cuda", dtype=torch.bfloat16)
    us = _time(lambda: C.gemm(a, b, out, False, False, 0, 1.0), warmup, iters)
    return f"gemm (CTA pair) {M}x{N}x{K}: {us:.1f} us, {2 * M * N * K / us / 1e6:.0f} TF/s"


def case_gemm_swiglu(warmup, iters):
    C = ext()
    M, N, K = B * S, 2 * I, H  # gate/up projection with the SwiGLU epilogue (training: saves gate/up)
    a = (torch.randn(M, K, device="cuda") * 0.05).to(torch.bfloat16)
    b = (torch.randn(N, K, device="cuda") * 0.05).to(torch.bfloat16)
    h = torch.empty(M, I, device="cuda", dtype=torch.bfloat16)
    gu = torch.empty(M, N, device="cuda", dtype=torch.bfloat16)
    us = _time(lambda: C.gemm(a, b, h, False, False, 5, 1.0, gu, I, I), warmup, iters)
    return f"gemm + SwiGLU epilogue (CTA pair) {M}x{N}x{K}: {us:.1f} us, {2 * M * N * K / us / 1e6:.0f} TF/s"


def case_gemm_residual(warmup, iters):
    C = ext()
    M, N, K = B * S, H, I  # down projection + residual
    a = (torch.randn(M, K, device="cuda") * 0.05).to(torch.bfloat16)
    b = (torch.randn(N, K, device="cuda") * 0.05).to(torch.bfloat16)
    r = torch.randn(M, N, device="cuda").to(torch.bfloat16)
    out = torch.empty(M, N, device="cuda", dtype=torch.bfloat16)
    us = _time(lambda: C.gemm(a, b, out, False, False, 1, 1.0, r), warmup, iters)
    return f"gemm + residual epilogue (CTA pair) {M}x{N}x{K}: {us:.1f} us, {2 * M * N * K / us / 1e6:.0f} TF/s"


def case_rmsnorm_bwd(warmup, iters):
    C = ext()
    T = B * S
    x, dy, dres = (torch.randn(T, H, device="cuda", dtype=torch.bfloat16) for _ in range(3))
    w = torch.randn(H, device="cuda", dtype=torch.bfloat16)
    rstd = torch.rand(T, device="cuda") + 0.5
    dx, dw = torch.empty_like(x), torch.zeros(H, device="cuda")
    us = _time(lambda: C.rmsnorm_bwd(dy, x, w, rstd, dx, dw, dres), warmup, iters)
    return f"rmsnorm bwd (+ residual grad) {T}x{H}: {us:.1f} us, {4 * T * H * 2 / us / 1e3:.0f} GB/s"


def case_qknorm(warmup, iters):
    C = ext()
    T = B * S
    qkv = torch.randn(T, (NQ + 2 * NKV) * D, device="cuda", dtype=torch.bfloat16)
    cos, sin = (torch.randn(S, D, device="cuda", dtype=torch.bfloat16) for _ in range(2))
    qw, kw = (torch.randn(D, device="cuda", dtype=torch.bfloat16) for _ in range(2))
    q = torch.empty(T, NQ * D, device="cuda", dtype=torch.bfloat16)
    k = torch.empty(T, NKV * D, device="cuda", dtype=torch.bfloat16)
    rstd = torch.empty(T * (NQ + NKV), device="cuda")
    us = _time(lambda: C.qknorm_rope_fwd(qkv, qw, kw, cos, sin, q, k, rstd, S, NQ, NKV, 1e-6), warmup, iters)
    return f"qk-norm + RoPE fwd {T} tokens x {NQ + NKV} heads: {us:.1f} us, {2 * T * (NQ + NKV) * D * 2 / us / 1e3:.0f} GB/s"


def case_qknorm_bwd(warmup, iters):
    C = ext()
    T = B * S
    nh = NQ + NKV
    qkv = torch.randn(T, (NQ + 2 * NKV) * D, device="cuda", dtype=torch.bfloat16)
    dq = torch.randn(T, NQ * D, device="cuda", dtype=torch.bfloat16)
    dk = torch.randn(T, NKV * D, device="cuda", dtype=torch.bfloat16)
    cos, sin = (torch.randn(S, D, device="cuda", dtype=torch.bfloat16) for _ in range(2))
    qw, kw = (torch.randn(D, device="cuda", dtype=torch.bfloat16) for _ in range(2))
    rstd = torch.rand(T * nh, device="cuda") + 0.5
    dqkv = torch.empty_like(qkv)
    dqw, dkw = torch.zeros(D, device="cuda"), torch.zeros(D, device="cuda")
    us = _time(lambda: C.qknorm_rope_bwd(dq, dk, qkv, qw, kw, cos, sin, rstd, dqkv, dqw, dkw, S, NQ, NKV),
               warmup, iters)
    moved = 3 * T * nh * D * 2  # gradient in, input rows in, input gradient out
    return f"qk-norm + RoPE bwd {T} tokens x {nh} heads: {us:.1f} us, {moved / us / 1e3:.0f} GB/s"


def case_wgrad_split(warmup, iters):
    """Weight-gradient GEMMs dW[M, N] = g^T x over T = B * S tokens at the
    0.6B step's split-K shapes: one K slice, split-K with fp32 atomics (zero
    fill + GEMM + cast) and the ordered split-K epilogue."""
    from .gemm import EPI_ATOMIC_F32, EPI_SPLIT_ORDERED, EPI_STORE_BF16, EPI_STORE_F32, _splitk

    C = ext()
    T = B * S
    lines = []
    for name, M, N in (("o_proj", H, NQ * D), ("gate_up", 2 * I, H), ("down", H, I), ("qkv", (NQ + 2 * NKV) * D, H)):
        g = torch.randn(T, M, device="cuda", dtype=torch.bfloat16)
        x = torch.randn(T, N, device="cuda", dtype=torch.bfloat16)
        out = torch.empty(M, N, device="cuda", dtype=torch.bfloat16)
        ws = torch.empty(M, N, device="cuda", dtype=torch.float32)
        sp = 2
        t1 = _time(lambda: C.gemm(g, x, out, True, True, EPI_STORE_BF16, 1.0), warmup, iters)

        def atomic():
            ws.zero_()
            C.gemm(g, x, ws, True, True, EPI_ATOMIC_F32, 1.0, splits=sp)
            C.cast_f32_to_bf16(ws, out)

        ta = _time(atomic, warmup, iters)
        to = _time(lambda: C.gemm(g, x, out, True, True, EPI_SPLIT_ORDERED, 1.0, splits=sp, ws=ws), warmup, iters)
        slabs = torch.empty(sp * M, N, device="cuda", dtype=torch.float32)

        def slab():
            C.gemm(g, x, slabs, True, True, EPI_STORE_F32, 1.0, splits=sp)
            C.sum_slices(slabs.view(sp, M * N), out.view(-1), False)

        tsl = _time(slab, warmup, iters)
        tf = 2 * M * N * T / 1e6
        lines.append(f"wgrad {name} {M}x{N}x{T}: 1 slice {t1:.1f} us ({tf / t1:.0f} TF/s), {sp} slices atomic+fill+cast "
                     f"{ta:.1f} us, {sp} slices ordered {to:.1f} us ({tf / to:.0f} TF/s), {sp} fp32 slabs + sum "
                     f"{tsl:.1f} us ({tf / tsl:.0f} TF/s); policy picks {_splitk(M, N, T)}")
    return "\n".join(lines)


def case_ce(warmup, iters):
    """Fused cross-entropy forward + gradient over one LM-head logits block
    (T = B * S rows of the 151,936-token vocabulary, gradient written in place):
    a statistics pass and a gradient pass per row; the algorithmic traffic is
    one read and one write of the logits."""
    C = ext()
    T, V = B * S, 151936
    logits = torch.randn(T, V, device="cuda", dtype=torch.bfloat16)
    labels = torch.randint(0, V, (T,), device="cuda")
    scale = torch.full((1,), 1.0 / T, device="cuda")
    lse, tgt = torch.empty(T, device="cuda"), torch.empty(T, device="cuda")
    us = _time(lambda: C.ce_fwd_bwd(logits, labels, 0, scale, lse, False, tgt, True), warmup, iters)
    return f"cross-entropy fwd+bwd {T}x{V}: {us:.1f} us, {2 * T * V * 2 / us / 1e3:.0f} GB/s"


def case_gemm_vs_cublas(warmup, iters):
    """Every GEMM of one Qwen3-0.6B training step (forward x W^T, input
    gradient g W, weight gradient g^T x for the five projections), this
    repository's CTA-pair kernel with the plain bf16 store against cuBLAS
    through torch.mm with the same operand layouts and a preallocated output."""
    from . import gemm as G

    T, V = B * S, 151936
    qkv = (NQ + 2 * NKV) * D
    layers = {"qkv": (qkv, H), "o_proj": (H, NQ * D), "gate_up": (2 * I, H), "down": (H, I), "lm_head": (V, H)}
    lines, tot = [], [0.0, 0.0, 0.0]
    for name, (n_out, k_in) in layers.items():
        w = (0.02 * torch.randn(n_out, k_in, device="cuda")).to(torch.bfloat16)
        x = torch.randn(T, k_in, device="cuda", dtype=torch.bfloat16)
        g = torch.randn(T, n_out, device="cuda", dtype=torch.bfloat16)
        # ours: the entry points the training step calls (they pick the tile
        # schedule: whole tiles, or split-K for few-tile long-K products)
        for kind, (M, N, K), ours, ref in (
                ("fwd", (T, n_out, k_in), lambda o: G.linear(x, w, out=o), lambda o: torch.mm(x, w.t(), out=o)),
                ("dgrad", (T, k_in, n_out), lambda o: G.linear_dgrad(g, w, out=o), lambda o: torch.mm(g, w, out=o)),
                ("wgrad", (n_out, k_in, T), lambda o: G.linear_wgrad(g, x, out=o),
                 lambda o: torch.mm(g.t(), x, out=o))):
            out = torch.empty(M, N, device="cuda", dtype=torch.bfloat16)
            t_ours = _time(lambda: ours(out), warmup, iters)
            t_ref = _time(lambda: ref(out), warmup, iters)
            tf = 2 * M * N * K / 1e6
            lines.append(f"{name:8s} {kind:5s} {M}x{N}x{K}: ours {t_ours:8.1f} us ({tf / t_ours:5.0f} TF/s)  "
                         f"cuBLAS {t_ref:8.1f} us ({tf / t_ref:5.0f} TF/s)  ratio {t_ref / t_ours:.2f}")
            tot[0] += t_ours * (28 if name != "lm_head" else 1)
            tot[1] += t_ref * (28 if name != "lm_head" else 1)
        del w, x, g
    lines.append(f"one step (28 layers + LM head): ours {tot[0] / 1e3:.2f} ms, cuBLAS {tot[1] / 1e3:.2f} ms")
    return "\n".join(lines)


def _oproj_wgrad_operands():
    T = B * S
    g = torch.randn(T, H, device="cuda", dtype=torch.bfloat16)
    x = torch.randn(T, NQ * D, device="cuda", dtype=torch.bfloat16)
    return g, x, torch.empty(H, NQ * D, device="cuda", dtype=torch.bfloat16)


def case_wgrad_oproj(warmup, iters):
    """The o_proj weight gradient (1024 x 2048 x 8192), one K slice, plain bf16
    store: the small case for profiler captures of the weight-gradient GEMM."""
    from .gemm import EPI_STORE_BF16

    C = ext()
    g, x, out = _oproj_wgrad_operands()
    us = _time(lambda: C.gemm(g, x, out, True, True, EPI_STORE_BF16, 1.0), warmup, iters)
    return f"wgrad o_proj one slice: {us:.1f} us, {2 * out.numel() * g.shape[0] / us / 1e6:.0f} TF/s"


def case_wgrad_oproj_cublas(warmup, iters):
    """The same product through cuBLAS (torch.mm with the same layouts)."""
    g, x, out = _oproj_wgrad_operands()
    us = _time(lambda: torch.mm(g.t(), x, out=out), warmup, iters)
    return f"wgrad o_proj cuBLAS: {us:.1f} us, {2 * out.numel() * g.shape[0] / us / 1e6:.0f} TF/s"


def case_moe_layer(warmup, iters):
    """One expert layer forward + backward at the per-rank shape of
    Qwen3-30B-A3B under EP = SP = 4 (32 local experts, hidden 2048, expert
    SwiGLU width 768, 8,192 routed rows, about 256 per expert): this
    repository's device-resident path (routing plan, dispatch into the padded
    expert matrix, tcgen05 grouped GEMMs with the SwiGLU epilogue, weighted
    combine; ``ops.moe.routed_experts``) against torch's composition (sort by
    expert, ``torch._grouped_mm``, SwiGLU, weights, unsort, sum over the
    top-k), the one the reference's HF expert modules run."""
    import torch.nn.functional as F

    from .moe import LocalExpertTransport, routed_experts

    E, Hd, Iw, T, K = 32, 2048, 768, 1024, 8
    g = torch.Generator(device="cpu").manual_seed(0)
    x = torch.randn(T, Hd, generator=g).to("cuda", torch.bfloat16).requires_grad_(True)
    sc, idx = torch.softmax(torch.randn(T, E, generator=g), -1).topk(K, -1)
    sc, idx = sc.cuda().requires_grad_(True), idx.cuda()
    w_gu = (torch.randn(E, 2 * Iw, Hd, generator=g) * 0.02).to("cuda", torch.bfloat16).requires_grad_(True)
    w_d = (torch.randn(E, Hd, Iw, generator=g) * 0.02).to("cuda", torch.bfloat16).requires_grad_(True)
    dout = torch.randn(T, Hd, generator=g).to("cuda", torch.bfloat16)
    transport = LocalExpertTransport(E)

    def ours():
        routed_experts(x, sc, idx, w_gu, w_d, transport).backward(dout)

    def torch_path():
        flat = idx.reshape(-1)
        order = torch.argsort(flat, stable=True)
        offs = torch.cumsum(torch.bincount(flat, minlength=E), 0).to(torch.int32)
        xs = x.repeat_interleave(K, 0).index_select(0, order)
        gu = torch._grouped_mm(xs, w_gu.transpose(1, 2), offs=offs)
        gt, up = gu.chunk(2, dim=-1)
        y = torch._grouped_mm((F.silu(gt) * up).contiguous(), w_d.transpose(1, 2), offs=offs)
        y = y * sc.reshape(-1)[order, None].to(y.dtype)
        out = torch.empty_like(y).index_copy_(0, order, y).view(T, K, Hd).sum(1)
        out.backward(dout)

    t_ours = _time(ours, warmup, iters)
    t_torch = _time(torch_path, warmup, iters)
    flops = 3 * 2 * T * K * Hd * 3 * Iw  # three products, forward + two backward
    from ..parallel.collective_bench import GEMM_PEAK as peak  # measured cuBLAS bf16 burst
    return (f"expert layer fwd+bwd ({T * K} routes, {E} experts, H {Hd}, I {Iw}): ours {t_ours:.1f} us "
            f"({flops / t_ours / 1e6:.0f} TF/s, {flops / t_ours / 1e6 / (peak / 1e12):.2f} of measured bf16), "
            f"torch._grouped_mm path {t_torch:.1f} us, speedup {t_torch / t_ours:.2f}x")


CASES = {"attn_fwd": case_attn_fwd, "moe_layer": case_moe_layer, "ce": case_ce, "gemm_vs_cublas": case_gemm_vs_cublas,
         "wgrad_oproj": case_wgrad_oproj, "wgrad_oproj_cublas": case_wgrad_oproj_cublas, "attn_bwd": case_attn_bwd, "gemm": case_gemm, "gemm_swiglu": case_gemm_swiglu,
         "gemm_residual": case_gemm_residual, "rmsnorm_bwd": case_rmsnorm_bwd, "qknorm": case_qknorm,
         "qknorm_bwd": case_qknorm_bwd, "wgrad_split": case_wgrad_split}


def main(argv=None):
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("case", choices=sorted(CASES) + ["all"])
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--iters", type=int, default=20)
    args = ap.parse_args(argv)
    torch.manual_seed(0)
    for name in (sorted(CASES) if args.case == "all" else [args.case]):
        print(CASES[name](args.warmup, args.iters), flush=True)


if __name__ == "__main__":
    main()
