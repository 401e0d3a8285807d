"""GPU test of the allocation-free attention backward entry point.

``pb_attention_bwd_noalloc`` is exported with C linkage from the extension
library for callers that cannot allocate device memory themselves; its
scratch lives in a fixed file-scope device array.  The test calls it through
its C symbol (ctypes), twice in a row, and compares dq / dk / dv with the
regular ``attn_bwd`` binding (which allocates its scratch through PyTorch),
using the tolerance of the other attention tests.  This file is named so that
pytest collects it last.
"""
import ctypes
import math

import pytest
import torch

pytestmark = pytest.mark.gpu


def _lib():
    import parallel_b200._C as C

    lib = ctypes.CDLL(C.__file__)
    fn = lib.pb_attention_bwd_noalloc
    fn.restype = ctypes.c_int
    fn.argtypes = ([ctypes.c_void_p] * 9 + [ctypes.c_int64] * 8 + [ctypes.c_int] * 5 + [ctypes.c_float, ctypes.c_int,
                                                                                         ctypes.c_void_p])
    lib.pb_attention_bwd_noalloc_last_error.restype = ctypes.c_char_p
    lib.pb_attention_bwd_noalloc_scratch_bytes.restype = ctypes.c_size_t
    lib.pb_attention_bwd_noalloc_device_status.restype = ctypes.c_int
    return C, lib, fn


def _rel(a, b):
    return ((a.float() - b.float()).norm() / (b.float().norm() + 1e-12)).item()


def _call(fn, q, k, v, o, do, lse, dq, dk, dv, B, S, nq, nkv, scale, causal):
    stream = torch.cuda.current_stream().cuda_stream
    return fn(q.data_ptr(), k.data_ptr(), v.data_ptr(), o.data_ptr(), do.data_ptr(), lse.data_ptr(), dq.data_ptr(),
              dk.data_ptr(), dv.data_ptr(), q.stride(0), k.stride(0), v.stride(0), o.stride(0), do.stride(0),
              dq.stride(0), dk.stride(0), dv.stride(0), B, S, nq, nkv, 128, scale, int(causal), stream)


# S = 200 ends partway through a 128-row tile, which exercises the padding of
# the per-row scratch and the bounds of the tiled loads
@pytest.mark.parametrize("causal", [True, False])
@pytest.mark.parametrize("S", [256, 200])
def test_noalloc_matches_allocating_entry_point(causal, S):
    C, lib, fn = _lib()
    torch.manual_seed(11)
    B, nq, nkv, D = 2, 4, 2, 128
    T = B * S
    scale = 1.0 / math.sqrt(D)
    q = torch.randn(T, nq * D, device="cuda").to(torch.bfloat16)
    k = torch.randn(T, nkv * D, device="cuda").to(torch.bfloat16)
    v = torch.randn(T, nkv * D, device="cuda").to(torch.bfloat16)
    o = torch.empty_like(q)
    lse = torch.zeros(B * nq * S + 128, device="cuda")
    C.attn_fwd(q, k, v, o, lse, B, S, nq, nkv, scale, causal)
    do = torch.randn_like(q)
    # regular (allocating) entry point
    delta = torch.empty(2 * (B * nq * S + 128), device="cuda")
    acc = torch.empty(T, nq * D, device="cuda")
    ref_dq, ref_dk, ref_dv = torch.empty_like(q), torch.empty_like(k), torch.empty_like(v)
    C.attn_bwd(q, k, v, o, do, lse, delta, acc, ref_dq, ref_dk, ref_dv, B, S, nq, nkv, scale, causal)
    lse_exact = lse[: B * nq * S].clone()  # no padding needed by the allocation-free variant
    for _ in range(2):
        dq, dk, dv = torch.full_like(q, 7.0), torch.full_like(k, 7.0), torch.full_like(v, 7.0)
        rc = _call(fn, q, k, v, o, do, lse_exact, dq, dk, dv, B, S, nq, nkv, scale, causal)
        assert rc == 0, lib.pb_attention_bwd_noalloc_last_error().decode()
        torch.cuda.synchronize()
        assert lib.pb_attention_bwd_noalloc_device_status() == 0
        assert _rel(dq, ref_dq) < 3e-2
        assert _rel(dk, ref_dk) < 3e-2
        assert _rel(dv, ref_dv) < 3e-2


def test_noalloc_rejects_oversized_problem():
    C, lib, fn = _lib()
    cap = lib.pb_attention_bwd_noalloc_scratch_bytes()
    B, S, nq, nkv = 1, 8192, 8, 8  # dq accumulator alone: 8192 * 1024 * 4 bytes = 32 MiB
    assert B * S * nq * 128 * 4 > cap
    t = torch.empty(8, device="cuda", dtype=torch.bfloat16)
    stream = torch.cuda.current_stream().cuda_stream
    rc = fn(*([t.data_ptr()] * 9), *([nq * 128] * 8), B, S, nq, nkv, 128, 0.088, 1, stream)
    assert rc == 1
    assert b"scratch" in lib.pb_attention_bwd_noalloc_last_error()
