"""Debug mode of the peer-memory data plane (``PB_COMM_DEBUG=1``): guard words
around symmetric buffers and span checks of peer launches, exercised on host
memory with a fake extension (no GPU needed; the checks are host code)."""
import pytest
import torch

from parallel_b200.parallel.comm import debug


@pytest.fixture(autouse=True)
def _fresh_registry():
    debug.clear()
    yield
    debug.clear()


def _region(name="bucket", payload=256, peer_ptrs=None):
    total, g = debug.guarded_numel(payload // 2, torch.bfloat16)
    raw = torch.zeros(total, dtype=torch.bfloat16).view(torch.uint8)
    base = raw.data_ptr() + g * 2
    reg = debug.register(debug.GuardedRegion(name, raw, g * 2, payload, peer_ptrs or [base, base + (1 << 30)]))
    return reg, base


def test_guarded_numel_keeps_a_fixed_byte_guard():
    assert debug.guarded_numel(1000, torch.bfloat16) == (1000 + 2 * 2048, 2048)
    assert debug.guarded_numel(1000, torch.float32) == (1000 + 2 * 1024, 1024)


def test_guard_words_detect_an_overrun_on_either_side():
    reg, _ = _region()
    reg.raw[reg.guard:reg.guard + reg.payload_bytes].fill_(7)   # payload writes are fine
    debug.check_canaries("ok")
    reg.raw[reg.guard + reg.payload_bytes + 3] = 0               # 4th byte past the end
    with pytest.raises(debug.CanaryViolation, match=r"'bucket' after payload \(byte 259\)"):
        debug.check_canaries("p2p_copy")
    reg.fill()
    reg.raw[reg.guard - 1] = 1                                   # last byte before the start
    with pytest.raises(debug.CanaryViolation, match=r"before payload \(byte -1\)"):
        debug.check_canaries("p2p_reduce")


def test_spans_must_stay_inside_the_payload_on_every_rank():
    reg, base = _region(payload=256)
    peer = reg.payload_ptrs[1]
    debug.check_spans("p2p_copy", [(base, 256), (peer + 128, 128)])
    debug.check_spans("p2p_copy", [(12345, 1 << 20)])             # not symmetric memory: not checked
    with pytest.raises(debug.PeerSpanError, match="rank 0"):
        debug.check_spans("p2p_copy", [(base + 128, 256)])         # runs past the end
    with pytest.raises(debug.PeerSpanError, match="rank 1"):
        debug.check_spans("p2p_copy", [(peer - 16, 32)])           # starts in the peer's guard


def test_checked_extension_validates_before_and_checks_guards_after():
    calls = []

    class Fake:
        def p2p_copy(self, src, dst, nbytes):
            calls.append(("copy", src, dst, nbytes))

        def p2p_reduce(self, src, dst, nelem, scale, accumulate):
            calls.append(("reduce", nelem))

        def gemm(self, *a):
            calls.append(("gemm",))
            return "plain"

    reg, base = _region(payload=256)
    C = debug.checked_extension(Fake())
    C.p2p_copy([base], [base + 128], [128])
    assert calls[-1][0] == "copy"
    with pytest.raises(debug.PeerSpanError):
        C.p2p_copy([base], [base + 192], [128])                   # destination overruns
    assert len(calls) == 1                                        # nothing launched
    with pytest.raises(debug.PeerSpanError):
        C.p2p_reduce([[base], [reg.payload_ptrs[1]]], [base + 64], [128], 0.5, False)  # 256 bytes from +64
    assert len(calls) == 1
    reg.raw[-1] = 0
    with pytest.raises(debug.CanaryViolation, match="after p2p_reduce"):
        C.p2p_reduce([[base]], [base], [64], 1.0, False)
    assert calls[-1] == ("reduce", [64])
    assert C.gemm() == "plain"                                    # non-peer launches pass through
