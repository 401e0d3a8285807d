"""Debug mode of the peer-memory data plane: guard words and span checks.

``PB_COMM_DEBUG=1`` switches it on (off by default; it synchronises the
device after every checked launch).  It finds the two errors that an
in-kernel collective can make without faulting: writing past the end of a
symmetric buffer (into a neighbouring allocation, on this GPU or a peer),
and being handed an address range that does not lie inside the buffer it
was meant for.

* **Guard words.** Every ``SymmBuffer`` is allocated with ``GUARD_BYTES`` on
  each side of its payload, filled with ``PATTERN``.  After each checked
  launch the device is synchronised and every rank compares the guards of
  its own buffers (a peer's overrun lands in this rank's memory, so the rank
  that owns the memory is the one that sees it) and raises
  ``CanaryViolation`` naming the buffer, the side and the first bad byte.
* **Span checks.** Before a peer copy / reduce launch, every (address,
  length) argument that starts inside a registered symmetric allocation
  (guards included, on any rank) must lie inside that allocation's payload;
  otherwise ``PeerSpanError`` is raised and nothing is launched.  Local
  tensors that are not symmetric are not checked here.
* ``checked_extension(mod)`` wraps the compiled extension so the peer
  launches go through both checks without changing their call sites.

The reference has no counterpart (it uses NCCL only; ordering safety comes
from stream discipline, parallel/parallel/engine/_dp_param_unit.py:353-361).
The peer protocols' own ordering is covered by epoch-numbered flags: a
stale flag never satisfies a wait for a newer epoch.
"""
from __future__ import annotations

import os
import weakref
from dataclasses import dataclass

import torch

GUARD_BYTES = 4096
PATTERN = 0xA5


def enabled() -> bool:
    return os.environ.get("PB_COMM_DEBUG", "0") == "1"


class CanaryViolation(RuntimeError):
    pass


class PeerSpanError(RuntimeError):
    pass


@dataclass
class GuardedRegion:
    """One symmetric allocation: ``raw`` is this rank's whole allocation as
    bytes (guard | payload | guard); ``payload_ptrs[r]`` is rank r's payload
    address as this process maps it."""

    name: str
    raw: torch.Tensor
    guard: int
    payload_bytes: int
    payload_ptrs: list

    def fill(self) -> None:
        self.raw[:self.guard].fill_(PATTERN)
        self.raw[self.guard + self.payload_bytes:].fill_(PATTERN)

    def bad_guards(self) -> list[tuple[str, int]]:
        out = []
        for side, seg, base in (("before", self.raw[:self.guard], 0),
                                ("after", self.raw[self.guard + self.payload_bytes:], self.guard + self.payload_bytes)):
            bad = (seg != PATTERN).nonzero()
            if bad.numel():
                out.append((side, base + int(bad[0, 0]) - self.guard))
        return out

    def locate(self, ptr: int):
        """(rank, payload start) of the allocation extent containing ``ptr``, or None."""
        for r, p in enumerate(self.payload_ptrs):
            if p - self.guard <= ptr < p + self.payload_bytes + self.guard:
                return r, p
        return None


_regions: list = []


def register(region: GuardedRegion) -> GuardedRegion:
    region.fill()
    _regions.append(weakref.ref(region))
    return region


def regions() -> list[GuardedRegion]:
    live = [w() for w in _regions]
    _regions[:] = [w for w, r in zip(_regions, live) if r is not None]
    return [r for r in live if r is not None]


def clear() -> None:
    _regions.clear()


def guarded_numel(numel: int, dtype: torch.dtype) -> tuple[int, int]:
    """(total elements to allocate, guard elements on each side)."""
    es = torch.empty(0, dtype=dtype).element_size()
    g = GUARD_BYTES // es
    return numel + 2 * g, g


def check_spans(op: str, spans) -> None:
    """``spans``: iterable of (address, nbytes)."""
    regs = regions()
    for ptr, n in spans:
        if n <= 0:
            continue
        for reg in regs:
            hit = reg.locate(ptr)
            if hit is None:
                continue
            r, p = hit
            if ptr < p or ptr + n > p + reg.payload_bytes:
                raise PeerSpanError(f"{op}: [{ptr:#x}, +{n}) leaves symmetric buffer '{reg.name}' of rank {r} "
                                    f"(payload [{p:#x}, +{reg.payload_bytes}))")
            break


def check_canaries(op: str) -> None:
    if torch.cuda.is_available() and torch.cuda.is_initialized():
        if torch.cuda.is_current_stream_capturing():
            return
        torch.cuda.synchronize()
    bad = [(reg.name, side, off) for reg in regions() for side, off in reg.bad_guards()]
    if bad:
        what = "; ".join(f"'{n}' {side} payload (byte {off})" for n, side, off in bad)
        raise CanaryViolation(f"after {op}: guard words overwritten: {what}")


def _spans_p2p_copy(src, dst, nbytes, *_):
    return list(zip(src, nbytes)) + list(zip(dst, nbytes))


def _spans_p2p_reduce(src, dst, nelem, *_):
    out = [(d, n * 2) for d, n in zip(dst, nelem)]
    for peer in src:
        out += [(s, n * 2) for s, n in zip(peer, nelem)]
    return out


_SPANS = {"p2p_copy": _spans_p2p_copy, "p2p_reduce": _spans_p2p_reduce}
# launches that move data between peers: guard words are checked after each
_PEER_OPS = ("p2p_copy", "p2p_reduce", "small_all_reduce", "gemm_ag", "gemm_rs", "row_gather", "row_gather_sum",
             "row_scatter")


class _CheckedExtension:
    def __init__(self, mod):
        self._mod = mod

    def __getattr__(self, name):
        fn = getattr(self._mod, name)
        if name not in _PEER_OPS:
            return fn
        spans = _SPANS.get(name)

        def checked(*args, **kwargs):
            if spans is not None:
                check_spans(name, spans(*args))
            out = fn(*args, **kwargs)
            check_canaries(name)
            return out

        return checked


def checked_extension(mod):
    return _CheckedExtension(mod)
