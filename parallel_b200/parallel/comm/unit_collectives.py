"""Data plane of the FSDP unit collectives (all-gather / reduce-scatter).

``TorchUnitCollectives`` runs them as ``torch.distributed`` collectives (NCCL
on GPUs, gloo on CPU) plus layout copies between the rank-major layout the
collectives use and the parameter-major layout the unit exposes.  It is the
CPU path and the measured NCCL baseline.  ``P2PUnitCollectives``
(``p2p.py``) does the same work with in-kernel NVLink peer loads on
symmetric memory and writes the parameter-major layout directly.
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import Any

import torch
import torch.distributed as dist

from ...profiling import collective_profile


def unit_detail(unit) -> str:
    return f"unit{unit.unit_index}:{unit.param_metas[0].name}+{len(unit.param_metas) - 1}params"


@dataclass
class _RSHandle:
    work: Any
    out: torch.Tensor
    grad_bucket: torch.Tensor
    accumulate: bool
    world: int
    keepalive: Any
    profile: Any


class TorchUnitCollectives:
    name = "nccl"

    def alloc_local_bucket(self, unit, numel: int, dtype, device) -> torch.Tensor:
        return torch.empty(numel, dtype=dtype, device=device)

    def release_full(self, unit, full: torch.Tensor) -> None:
        pass

    # ---------------------------------------------------------------- gather
    def all_gather(self, unit, mode: str = "demand") -> torch.Tensor:
        N, nb = unit.world_size, unit.bucket_numel
        src = unit.local_bucket
        if src.device != unit.device:
            src = src.to(unit.device, non_blocking=True)
        tmp = torch.empty(N * nb, dtype=src.dtype, device=unit.device)
        with collective_profile("fsdp_all_gather", value=src, mode=mode, detail=unit_detail(unit)):
            dist.all_gather_into_tensor(tmp, src, group=unit.group)
        full = torch.empty(unit.full_numel, dtype=src.dtype, device=unit.device)
        tv = tmp.view(N, nb)
        for m in unit.param_metas:
            full.narrow(0, m.full_offset, N * m.padded_numel).view(N, m.padded_numel).copy_(
                tv[:, m.bucket_offset:m.bucket_offset + m.padded_numel])
        return full

    # ---------------------------------------------------------------- reduce
    @staticmethod
    def pack_rank_major(unit, grads) -> torch.Tensor:
        """[N, bucket] rank-major reduce-scatter input from full gradients."""
        N, nb = unit.world_size, unit.bucket_numel
        tmp = torch.zeros(N, nb, dtype=unit.local_bucket.dtype, device=unit.device)
        for g, m in zip(grads, unit.param_metas):
            if g is None:
                continue
            g2 = g.reshape(m.shape[0], -1)
            if g2.dtype != tmp.dtype:
                g2 = g2.to(tmp.dtype)
            if m.shape[0] == N * m.padded_rows:
                tmp[:, m.bucket_offset:m.bucket_offset + m.padded_numel].copy_(g2.reshape(N, m.padded_numel))
                continue
            for r in range(N):
                s = r * m.padded_rows
                rows = min(m.padded_rows, max(m.shape[0] - s, 0))
                if rows:
                    tmp[r, m.bucket_offset:m.bucket_offset + rows * m.row_numel].copy_(
                        g2[s:s + rows].reshape(-1))
        return tmp

    def reduce_scatter(self, unit, grads, grad_bucket, accumulate: bool, mode: str = "overlapped"):
        tmp = self.pack_rank_major(unit, grads)
        out = torch.empty_like(grad_bucket) if accumulate else grad_bucket
        prof = collective_profile("fsdp_reduce_scatter", value=tmp, mode=mode, detail=unit_detail(unit),
                                  defer_cuda_end=True)
        with prof:
            work = dist.reduce_scatter_tensor(out, tmp.view(-1), op=dist.ReduceOp.SUM, group=unit.group,
                                              async_op=True)
        return _RSHandle(work, out, grad_bucket, accumulate, unit.world_size, tmp, prof)

    def wait(self, h: _RSHandle) -> None:
        h.work.wait()
        h.profile.complete()
        h.out.div_(h.world)
        if h.accumulate:
            h.grad_bucket.add_(h.out)
        h.keepalive = None


def make_unit_collectives(kind: str, device: torch.device, group=None):
    """``auto`` picks the NVLink P2P kernels on CUDA when they are available."""
    kind = (kind or "auto").lower()
    if device.type != "cuda" or kind == "nccl":
        return TorchUnitCollectives()
    if kind in ("auto", "p2p"):
        try:
            from .p2p import P2PUnitCollectives, p2p_supported
        except ImportError:
            if kind == "p2p":
                raise
            return TorchUnitCollectives()
        if p2p_supported(group):
            return P2PUnitCollectives(group)
        if kind == "p2p":
            raise RuntimeError("P2P collectives requested but symmetric memory is unavailable")
    return TorchUnitCollectives()
