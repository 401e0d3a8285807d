"""Matrix products on the tcgen05 GEMM (``csrc/gemm.cu``).

Three layouts cover every nn.Linear product of training without transposes:

* ``linear(x, w)``      = x @ w.T      (forward;  A, B K-major)
* ``linear_dgrad(g, w)`` = g @ w        (input grad; B MN-major)
* ``linear_wgrad(g, x)`` = g.T @ x      (weight grad; A, B MN-major)

On CUDA tensors the native kernel runs (and must be built); on CPU tensors a
PyTorch restatement runs in the tensor's dtype with fp32 accumulation, which
is what the CPU parity tests use.
"""
from __future__ import annotations

import torch

from ._ext import ext, use_kernels

EPI_STORE_BF16 = 0
EPI_RESIDUAL_BF16 = 1
EPI_STORE_F32 = 2
EPI_ACCUM_BF16 = 3
EPI_ACCUM_F32 = 4
EPI_SWIGLU = 5
EPI_ATOMIC_F32 = 6
EPI_SPLIT_ORDERED = 7

# Split-K for long-K products with few CTA-pair tiles (the weight gradients
# reduce over all tokens).  Each K slice writes its fp32 partial tile into its
# own slab with TMA tile stores and one pass adds the slabs in slice order (no
# waits between slices, no atomics, the same bits on every run).  The slice
# count minimises a wave model: ceil(tiles * s / pairs) / s waves of the unsplit
# tile time, plus the slab round trip (write and read of s fp32 partials).
# Measured on B200 at T = 8192, the o_proj weight gradient (1024 x 2048, 32
# tiles on 74 SM pairs) is the step's product that gains; the ordered split-K
# (each slice waiting for the previous one's running sum) lost on every shape.
_SPLITK_MIN_K = 2048
_PAIR_TFLOPS = 22e12    # one SM pair's bf16 rate inside a long-K tile (measured ~0.7 of peak)
_SLAB_BYTES_PER_S = 5e12


def _pair_slots() -> int:
    try:
        return max(1, torch.cuda.get_device_properties(torch.cuda.current_device()).multi_processor_count // 2)
    except Exception:
        return 74


def _splitk(M: int, N: int, K: int, slots: int | None = None) -> int:
    if M < 256 or K < 2 * _SPLITK_MIN_K:
        return 1
    slots = slots or _pair_slots()
    tiles = ((M + 255) // 256) * ((N + 255) // 256)
    t_tile = 2.0 * 256 * 256 * K / _PAIR_TFLOPS

    def cost(s):
        waves = -(-tiles * s // slots) / s
        slab = 0.0 if s == 1 else 2.0 * s * M * N * 4 / _SLAB_BYTES_PER_S
        return waves * t_tile + slab

    best = 1
    for s in (2, 3, 4):
        if K // s >= _SPLITK_MIN_K and cost(s) < 0.9 * cost(best):
            best = s
    return best


def _rows(t: torch.Tensor) -> torch.Tensor:
    return t.reshape(-1, t.shape[-1])


def linear(x: torch.Tensor, w: torch.Tensor, residual: torch.Tensor | None = None,
           out: torch.Tensor | None = None) -> torch.Tensor:
    """``x @ w.T (+ residual)`` for x [..., K], w [N, K]."""
    lead = x.shape[:-1]
    x2 = _rows(x)
    if not use_kernels(x2):
        y = (x2.float() @ w.float().t())
        if residual is not None:
            y = y + _rows(residual).float()
        return y.to(x.dtype).reshape(*lead, w.shape[0])
    x2 = x2 if x2.stride(-1) == 1 else x2.contiguous()
    if out is None:
        out = torch.empty(x2.shape[0], w.shape[0], dtype=torch.bfloat16, device=x.device)
    if residual is not None:
        ext().gemm(x2, w, out, False, False, EPI_RESIDUAL_BF16, 1.0, _rows(residual))
    else:
        ext().gemm(x2, w, out, False, False, EPI_STORE_BF16, 1.0)
    return out.reshape(*lead, w.shape[0])


def linear_swiglu(x: torch.Tensor, w_gate_up: torch.Tensor, inter: int,
                  save_gu: bool = True) -> tuple[torch.Tensor, torch.Tensor | None]:
    """``silu(x @ Wg.T) * (x @ Wu.T)`` with Wg = w[:inter], Wu = w[inter:2*inter].

    Returns (h [T, inter], gu [T, 2*inter] or None) where gu holds the bf16
    gate/up pre-activations needed by the backward.
    """
    x2 = _rows(x)
    if not use_kernels(x2):
        gu = (x2.float() @ w_gate_up.float().t()).to(x.dtype)
        g, u = gu[:, :inter], gu[:, inter:]
        h = (torch.nn.functional.silu(g.float()).to(x.dtype).float() * u.float()).to(x.dtype)
        return h, (gu if save_gu else None)
    T = x2.shape[0]
    h = torch.empty(T, inter, dtype=torch.bfloat16, device=x.device)
    gu = torch.empty(T, 2 * inter, dtype=torch.bfloat16, device=x.device) if save_gu else None
    ext().gemm(x2, w_gate_up, h, False, False, EPI_SWIGLU, 1.0, gu, inter, inter)
    return h, gu


def linear_dgrad(g: torch.Tensor, w: torch.Tensor, out: torch.Tensor | None = None,
                 accumulate: bool = False) -> torch.Tensor:
    """``g @ w`` for g [T, N], w [N, K] -> [T, K]."""
    g2 = _rows(g)
    if not use_kernels(g2):
        y = g2.float() @ w.float()
        if accumulate and out is not None:
            out.add_(y.to(out.dtype))
            return out
        return y.to(g.dtype)
    g2 = g2 if g2.stride(-1) == 1 else g2.contiguous()
    if out is None:
        out = torch.empty(g2.shape[0], w.shape[1], dtype=torch.bfloat16, device=g.device)
        accumulate = False
    epi = EPI_ACCUM_BF16 if accumulate else EPI_STORE_BF16
    if out.dtype == torch.float32:
        epi = EPI_ACCUM_F32 if accumulate else EPI_STORE_F32
    ext().gemm(g2, w, out, False, True, epi, 1.0)
    return out


def linear_wgrad(g: torch.Tensor, x: torch.Tensor, out: torch.Tensor | None = None,
                 accumulate: bool = False, out_dtype: torch.dtype = torch.bfloat16) -> torch.Tensor:
    """``g.T @ x`` for g [T, N], x [T, K] -> [N, K]."""
    g2, x2 = _rows(g), _rows(x)
    if not use_kernels(g2):
        y = g2.float().t() @ x2.float()
        if out is not None:
            if accumulate:
                out.add_(y.to(out.dtype))
            else:
                out.copy_(y)
            return out
        return y.to(out_dtype)
    g2 = g2 if g2.stride(-1) == 1 else g2.contiguous()
    x2 = x2 if x2.stride(-1) == 1 else x2.contiguous()
    if out is None:
        out = torch.empty(g2.shape[1], x2.shape[1], dtype=out_dtype, device=g.device)
        accumulate = False
    M, N, K = g2.shape[1], x2.shape[1], g2.shape[0]
    splits = _splitk(M, N, K)
    if splits > 1 and out.is_contiguous():
        # split-K over the tokens: slice s stores its fp32 partial in slab s,
        # then the slabs are added in slice order into out (bf16 or fp32,
        # optionally accumulating)
        slabs = torch.empty(splits * M, N, dtype=torch.float32, device=g.device)
        ext().gemm(g2, x2, slabs, True, True, EPI_STORE_F32, 1.0, splits=splits)
        ext().sum_slices(slabs.view(splits, M * N), out.view(-1), accumulate)
        return out
    if out.dtype == torch.float32:
        epi = EPI_ACCUM_F32 if accumulate else EPI_STORE_F32
    else:
        epi = EPI_ACCUM_BF16 if accumulate else EPI_STORE_BF16
    ext().gemm(g2, x2, out, True, True, epi, 1.0)
    return out


def gemm_raw(a: torch.Tensor, b: torch.Tensor, out: torch.Tensor, a_mn: bool, b_mn: bool,
             epi: int = EPI_STORE_BF16, alpha: float = 1.0, r: torch.Tensor | None = None) -> torch.Tensor:
    """Direct access to the kernel (tests / benchmarks)."""
    ext().gemm(a, b, out, a_mn, b_mn, epi, alpha, r)
    return out
