"""NVLink peer-to-peer data plane for FSDP units (symmetric memory + own kernels).

Every FSDP local bucket and the reduce-scatter staging slots are allocated
as symmetric memory (``torch.distributed._symmetric_memory``: one mapping of
every peer's buffer per process; used here only for allocation and handle
exchange).  The data movement is done by this repository's kernels
(``csrc/comm.cu``):

* all-gather: one bounded signal barrier ("my shard is current"), then one
  kernel that loads every peer's shard over NVLink and stores it straight
  into the parameter-major full buffer (no rank-major staging, no unpack);
* reduce-scatter: gradients are packed into a symmetric slot, one barrier
  ("my gradients are staged"), one kernel that sums the rank's shard rows
  from all peers in fp32 and writes (or accumulates into) the local bf16
  gradient bucket scaled by 1/N; it runs on a dedicated communication stream
  so it overlaps the next unit's backward.  A slot is restaged only after the
  barrier of the following reduction has passed (every rank finished reading
  it), which needs no closing barrier.

Barriers are bounded (``PB_P2P_TIMEOUT_S``, default 60 s): a missing peer
records an error word on the device instead of hanging; the engine reads it
asynchronously and raises ``CollectiveTimeout``.
"""
from __future__ import annotations

import importlib
import os
from dataclasses import dataclass
from typing import Any

import torch
import torch.distributed as dist

from ...ops._ext import ext
from ...profiling import collective_profile
from . import debug as comm_debug
from .unit_collectives import TorchUnitCollectives, unit_detail


class CollectiveTimeout(RuntimeError):
    pass


def p2p_supported(group) -> bool:
    if os.environ.get("PB_P2P", "1") == "0":
        return False
    if group is None or not torch.cuda.is_available():
        return False
    try:
        importlib.import_module("torch.distributed._symmetric_memory")
    except ImportError:
        return False
    return 1 < dist.get_world_size(group) <= 8


class SymmBuffer:
    """A symmetric allocation plus its peer addresses and signal pads."""

    def __init__(self, numel: int, dtype, device, group, name: str = "symm"):
        symm_mem = importlib.import_module("torch.distributed._symmetric_memory")
        numel = max(numel, 64)
        # debug mode: guard words on both sides of the payload (same on every rank)
        total, guard = comm_debug.guarded_numel(numel, dtype) if comm_debug.enabled() else (numel, 0)
        self._alloc = symm_mem.empty(total, dtype=dtype, device=device)
        self.tensor = self._alloc[guard:guard + numel] if guard else self._alloc
        self.tensor.zero_()
        self.handle = symm_mem.rendezvous(self._alloc, group)
        self.rank = self.handle.rank
        self.world = self.handle.world_size
        base = list(self.handle.buffer_ptrs)
        off = self.tensor.data_ptr() - base[self.rank]
        self.peer_ptrs = [b + off for b in base]
        self.guard = None
        if guard:
            es = self.tensor.element_size()
            self.guard = comm_debug.register(comm_debug.GuardedRegion(
                name, self._alloc.view(torch.uint8), guard * es, numel * es, list(self.peer_ptrs)))
        self.pads_dev = int(self.handle.signal_pad_ptrs_dev)
        # per-channel epoch counters live on the device: the barrier kernel bumps
        # them, so a captured CUDA graph that contains barriers replays correctly
        self.epochs = torch.zeros(8, dtype=torch.int32, device=device)
        self.event = None

    def barrier(self, channel: int, limit_s: float) -> None:
        ext().p2p_barrier(self.pads_dev, self.rank, self.world, channel * 8, self.epochs, channel, limit_s)


class P2PSmallAllReduce:
    """All-reduce of small fp32 vectors over NVLink peer memory in one kernel
    (``csrc/comm.cu``: each block pushes its slice into every peer's symmetric
    region, raises a per-block device epoch flag and sums its slice locally;
    two parities of slots, no closing barrier, CUDA-graph safe).  Used for the
    gradient-norm / finite-flag reductions, the load-balancing-loss statistics
    and the vocab-parallel log-sum-exp merge instead of NCCL all-reduces.

    ``get(group, device)`` returns the instance of a group (creating it is
    collective: every rank of the group must make the first call together)."""

    _instances: dict = {}
    MAX_BLOCKS = 64

    def __init__(self, group, device, cap_units: int = 16384):
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        self.cap = cap_units
        self.limit_s = float(os.environ.get("PB_P2P_TIMEOUT_S", "60"))
        self.buf = SymmBuffer(ext().small_ar_region_floats(self.world, cap_units), torch.float32, device, group,
                              "small_all_reduce")
        self.bases = list(self.buf.peer_ptrs)
        self.epochs = torch.zeros(self.MAX_BLOCKS, dtype=torch.int32, device=device)

    @classmethod
    def get(cls, group, device):
        if not (device.type == "cuda" and p2p_supported(group)):
            return None
        key = (id(group), device.index)
        inst = cls._instances.get(key)
        if inst is None:
            inst = cls._instances[key] = cls(group, device)
        return inst

    def _run(self, x: torch.Tensor, out: torch.Tensor, units: int, op: int) -> None:
        ext().small_all_reduce(x, out, units, op, self.bases, self.rank, self.cap, self.epochs, self.limit_s)

    def all_reduce_(self, t: torch.Tensor, op: str = "sum") -> torch.Tensor:
        """In-place SUM / MAX of an fp32 CUDA tensor (at most 3 x cap elements)."""
        if t.dtype != torch.float32 or not t.is_contiguous():
            raise TypeError("P2PSmallAllReduce works on contiguous fp32 tensors")
        if t.numel() > 3 * self.cap:
            raise ValueError(f"{t.numel()} elements exceed the {3 * self.cap}-element buffer")
        self._run(t, t, t.numel(), {"sum": 0, "max": 1}[op])
        return t

    def lse_merge(self, row_max: torch.Tensor, row_sumexp: torch.Tensor, row_target: torch.Tensor):
        """Global (log-sum-exp, target) per row from every rank's local row max,
        sum of exp(x - local max) and target-logit contribution."""
        rows = row_max.numel()
        if rows > self.cap:
            raise ValueError(f"{rows} rows exceed the {self.cap}-row buffer")
        packed = torch.stack([row_max.float(), row_sumexp.float(), row_target.float()]).contiguous()
        out = torch.empty(2, rows, device=packed.device, dtype=torch.float32)
        self._run(packed, out, rows, 2)
        return out[0], out[1]


class ReplicaMeanAllReduce:
    """Mean of a fixed list of bf16 gradient buffers over the dp_replicate
    group on NVLink peer memory (the reference all-reduces each gradient with
    NCCL, parallel/parallel/engine/engine.py:224-247).

    One-shot scheme: every rank copies its buffers into its slot of a
    symmetric staging region (one multi-segment copy kernel), a signal barrier
    publishes them, and one kernel per 16 buffers sums the R replicas' slots
    in fp32, scales by 1/R and writes the local buffers.  Each rank reads the
    other replicas' full buffers over NVLink (R - 1 copies, what a ring
    all-reduce moves for R <= 2 and close to it for R <= 4) with a single
    barrier and no reduce-scatter / all-gather phases.  Two staging sets
    rotate; a rank writes a set only after the barrier of the call in between,
    which every rank reaches after its reads of the set's previous use.
    Buffers must be bf16 CUDA, contiguous, 16-byte aligned and a multiple of 8
    elements (``eligible``); the sizes are fixed by the first call."""

    _instances: dict = {}

    def __init__(self, group, device, sizes: tuple[int, ...]):
        self.group = group
        self.world = dist.get_world_size(group)
        self.sizes = sizes
        self.offsets, off = [], 0
        for n in sizes:
            self.offsets.append(off)
            off += -(-n // 8) * 8
        self.limit_s = float(os.environ.get("PB_P2P_TIMEOUT_S", "60"))
        self.nvls = NvlsAllReduce.get(group, device, off)
        self.sets = [] if self.nvls is not None else [
            SymmBuffer(max(off, 8), torch.bfloat16, device, group, "replica_grads") for _ in range(2)]
        self.turn = 0

    @staticmethod
    def eligible(tensors) -> bool:
        return bool(tensors) and all(t.is_cuda and t.dtype == torch.bfloat16 and t.is_contiguous()
                                     and t.numel() % 8 == 0 and t.data_ptr() % 16 == 0 for t in tensors)

    @classmethod
    def get(cls, group, device, tensors):
        """The instance for this group and buffer layout (creating it is
        collective over the group), or None when peer memory or the buffers
        do not qualify."""
        if not (device.type == "cuda" and p2p_supported(group) and cls.eligible(tensors)):
            return None
        sizes = tuple(t.numel() for t in tensors)
        key = (id(group), device.index, sizes)
        if key not in cls._instances:
            cls._instances[key] = cls(group, device, sizes)
        return cls._instances[key]

    def mean_(self, tensors) -> None:
        if self.nvls is not None:
            self.nvls.all_reduce_(tensors, 1.0 / self.world)
            return
        buf = self.sets[self.turn % 2]
        self.turn += 1
        base = buf.tensor.data_ptr()
        ext().p2p_copy([t.data_ptr() for t in tensors], [base + 2 * o for o in self.offsets],
                       [2 * t.numel() for t in tensors])
        buf.barrier(0, self.limit_s)
        srcs = [[p + 2 * o for o in self.offsets] for p in buf.peer_ptrs]
        ext().p2p_reduce(srcs, [t.data_ptr() for t in tensors], [t.numel() for t in tensors], 1.0 / self.world,
                         False)


def nvls_mode() -> str:
    """``PB_NVLS``: ``0`` never uses the in-switch all-reduce, ``1`` uses it
    wherever the probe passes, ``auto`` (default) as ``1`` for groups of
    more than two ranks, where it halves the NVLink traffic of the peer-load
    all-reduce (at two ranks both move the same bytes)."""
    return os.environ.get("PB_NVLS", "auto")


class NvlsAllReduce:
    """All-reduce of bf16 buffers through the NVSwitch (NVLS): the symmetric
    staging buffer is bound to an NVLink multicast object, every rank reduces
    its 1/world slice with ``multimem.ld_reduce`` (the switch sums all GPUs'
    copies, fp32 accumulation) and writes the result to every GPU with one
    ``multimem.st`` (``csrc/comm.cu``).  Each GPU then receives every byte once,
    where the peer-load scheme (owners pull and sum, then everyone gathers)
    receives it 2 (world - 1) / world times.

    Capability probe (``get``): the device reports switch multicast
    (``CU_DEVICE_ATTRIBUTE_MULTICAST_SUPPORTED``), every rank of the group
    agrees, and the symmetric allocation came back with a multicast address;
    otherwise None and the caller keeps its peer-load path.  The reference
    all-reduces with NCCL (parallel/parallel/engine/engine.py:224-247), which
    picks NVLS itself when the fabric offers it.

    Staging: copy in, barrier, reduce + broadcast, barrier, copy out.  After
    the second barrier no rank reads or writes another's buffer any more, so
    one buffer serves every call."""

    _instances: dict = {}

    def __init__(self, group, device, capacity: int):
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        self.capacity = -(-capacity // 8) * 8
        self.limit_s = float(os.environ.get("PB_P2P_TIMEOUT_S", "60"))
        self.buf = SymmBuffer(self.capacity, torch.bfloat16, device, group, "nvls_all_reduce")
        # the multicast mapping covers the allocation from its base (the handle's
        # own buffer pointer); the payload starts `off` bytes in (guard words in
        # the debug mode) and must end inside it
        h = self.buf.handle
        mc = int(getattr(h, "multicast_ptr", 0) or 0)
        off = self.buf.tensor.data_ptr() - int(list(h.buffer_ptrs)[self.rank])
        inside = int(getattr(h, "offset", 0) or 0) == 0 and 0 <= off and off + 2 * self.capacity <= int(h.buffer_size)
        self.mc = mc + off if (mc and inside) else 0

    @staticmethod
    def probe(group, device) -> bool:
        """True on every rank when every rank's device supports switch
        multicast (collective over ``group``; CUDA devices only)."""
        if device.type != "cuda" or not p2p_supported(group):
            return False
        ok = torch.tensor([1 if ext().device_multicast_supported(device.index) else 0], device=device,
                          dtype=torch.int32)
        dist.all_reduce(ok, op=dist.ReduceOp.MIN, group=group)
        return bool(ok.item())

    @classmethod
    def get(cls, group, device, capacity: int, force: bool = False):
        """The group's instance holding at least ``capacity`` elements, or
        None when NVLS is off (``PB_NVLS``) or not available.  Creating it is
        collective over the group."""
        mode = nvls_mode()
        world = dist.get_world_size(group)
        if device.type != "cuda" or mode == "0" or (mode == "auto" and world <= 2 and not force):
            return None
        key = (id(group), device.index)
        inst = cls._instances.get(key)
        if inst is not None and inst.capacity >= capacity:
            return inst if inst.mc else None
        if torch.cuda.is_current_stream_capturing():  # the probe and the allocation are host-synchronous
            return None
        if not cls.probe(group, device):
            return None
        inst = cls(group, device, capacity)
        ok = torch.tensor([1 if inst.mc else 0], device=device, dtype=torch.int32)
        dist.all_reduce(ok, op=dist.ReduceOp.MIN, group=group)
        if not ok.item():
            inst.mc = 0
        cls._instances[key] = inst
        return inst if inst.mc else None

    def all_reduce_(self, tensors, scale: float = 1.0, outs=None) -> None:
        """Each bf16 tensor's scale x sum over the group, written in place or
        into ``outs`` (same shapes).  Tensors are contiguous, 16-byte aligned,
        a multiple of 8 elements and together at most ``capacity`` elements."""
        outs = tensors if outs is None else outs
        offs, off = [], 0
        for t in tensors:
            offs.append(off)
            off += t.numel()
        if off > self.capacity:
            raise ValueError(f"{off} elements exceed the {self.capacity}-element NVLS buffer")
        base = self.buf.tensor.data_ptr()
        ext().p2p_copy([t.data_ptr() for t in tensors], [base + 2 * o for o in offs],
                       [2 * t.numel() for t in tensors])
        self.buf.barrier(0, self.limit_s)
        ext().multimem_all_reduce(self.mc, off, self.rank, self.world, scale)
        self.buf.barrier(1, self.limit_s)
        ext().p2p_copy([base + 2 * o for o in offs], [t.data_ptr() for t in outs],
                       [2 * t.numel() for t in tensors])


@dataclass
class _P2PHandle:
    event: Any
    profile: Any
    torch_handle: Any = None


class P2PUnitCollectives:
    name = "p2p"

    def __init__(self, group):
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        self.limit_s = float(os.environ.get("PB_P2P_TIMEOUT_S", "60"))
        self.slots: list[SymmBuffer] = []
        self._slot_numel = 0
        self._next_slot = 0
        self.stream = None
        self._need_barrier = True
        self._prev_slot = None
        self._fallback = TorchUnitCollectives()

    # ------------------------------------------------------------ allocation
    @staticmethod
    def _aligned(unit) -> bool:
        es = unit.param_metas[0].parameter.element_size()
        return es == 2 and all((m.padded_numel * es) % 16 == 0 for m in unit.param_metas)

    def alloc_local_bucket(self, unit, numel, dtype, device):
        if not self._aligned(unit):
            unit._p2p = None
            return self._fallback.alloc_local_bucket(unit, numel, dtype, device)
        buf = SymmBuffer(numel, dtype, device, self.group, "fsdp_bucket")
        unit._p2p = buf
        return buf.tensor[:numel]

    def release_full(self, unit, full):
        pass

    def reset_step_events(self) -> None:
        """Forget the slot-reuse events of finished steps.  Valid between steps:
        the gradient-norm all-reduce that ends a step follows every rank's
        reductions, so every slot is free when the next step starts (needed
        before a CUDA-graph capture, which cannot wait on earlier events)."""
        for s in self.slots:
            s.event = None
        self._prev_slot = None

    def begin_forward(self) -> None:
        """A forward pass starts: the shards may have changed since the last
        one (optimizer step, checkpoint load), so the first all-gather waits
        for every rank once.  Within the pass the shards are read-only, and
        every rank finishes its reads of pass k before it can update its shard
        (the optimizer step follows the gradient-norm all-reduce), so the
        later gathers need no barrier."""
        self._need_barrier = True

    # ------------------------------------------------------------ all-gather
    def all_gather(self, unit, mode: str = "demand") -> torch.Tensor:
        buf = getattr(unit, "_p2p", None)
        if buf is None:
            return self._fallback.all_gather(unit, mode)
        es = 2
        full = torch.empty(unit.full_numel, dtype=unit.local_bucket.dtype, device=unit.device)
        src, dst, nb = [], [], []
        fbase = full.data_ptr()
        # each rank starts with its own shard and walks the peers from rank+1:
        # the copy kernel's blocks run roughly in segment order, and a common
        # order would have every rank read the same source's NVLink port at once
        for i in range(self.world):
            r = (self.rank + i) % self.world
            for m in unit.param_metas:
                if m.padded_numel == 0:
                    continue
                src.append(buf.peer_ptrs[r] + m.bucket_offset * es)
                dst.append(fbase + (m.full_offset + r * m.padded_numel) * es)
                nb.append(m.padded_numel * es)
        with collective_profile("fsdp_all_gather", value=unit.local_bucket, mode=mode, detail=unit_detail(unit)):
            if self._need_barrier:
                buf.barrier(0, self.limit_s)
                self._need_barrier = False
            ext().p2p_copy(src, dst, nb)
        return full

    # ------------------------------------------------------------ reduce-scatter
    def _slot(self, unit) -> SymmBuffer:
        if not self.slots:
            raise RuntimeError("reduce-scatter slots not allocated")
        s = self.slots[self._next_slot % len(self.slots)]
        self._next_slot += 1
        return s

    def prepare(self, units) -> None:
        """Allocate the reduce-scatter staging slots (collective; call once)."""
        need = max((u.full_numel for u in units if getattr(u, "_p2p", None) is not None), default=0)
        if need == 0 or self.slots:
            return
        dev = units[0].device
        self._slot_numel = need
        self.slots = [SymmBuffer(need, torch.bfloat16, dev, self.group, "fsdp_rs_slot") for _ in range(3)]
        self.stream = torch.cuda.Stream(device=dev)

    def reduce_scatter(self, unit, grads, grad_bucket, accumulate: bool, mode: str = "overlapped"):
        buf = getattr(unit, "_p2p", None)
        if buf is None or not self.slots:
            return _P2PHandle(None, None, self._fallback.reduce_scatter(unit, grads, grad_bucket, accumulate, mode))
        slot = self._slot(unit)
        cur = torch.cuda.current_stream(unit.device)
        if slot.event is not None:  # every rank is done reading this slot's previous contents
            cur.wait_event(slot.event)
        N = self.world
        st = slot.tensor
        for g, m in zip(grads, unit.param_metas):
            rows = N * m.padded_rows
            view = st.narrow(0, m.full_offset, rows * m.row_numel).view(rows, -1)
            if g is None:
                view.zero_()
                continue
            g2 = g.reshape(m.shape[0], -1)
            view[: m.shape[0]].copy_(g2)
            if m.shape[0] < rows:
                view[m.shape[0]:].zero_()
        self.stream.wait_stream(cur)
        es = 2
        src = [[slot.peer_ptrs[r] + (m.full_offset + self.rank * m.padded_numel) * es for m in unit.param_metas]
               for r in range(N)]
        dst = [grad_bucket.data_ptr() + m.bucket_offset * es for m in unit.param_metas]
        nel = [m.padded_numel for m in unit.param_metas]
        prof = collective_profile("fsdp_reduce_scatter", payload_bytes=unit.full_numel * es, mode=mode,
                                  detail=unit_detail(unit), device=unit.device, defer_cuda_end=True)
        with torch.cuda.stream(self.stream):
            with prof:
                # every rank has staged its gradients into its slot
                slot.barrier(1, self.limit_s)
                # ...which also means every rank finished the previous reduction
                # (issued before this barrier on its side stream), so the
                # previous slot may be restaged
                if self._prev_slot is not None:
                    freed = torch.cuda.Event()
                    freed.record(self.stream)
                    self._prev_slot.event = freed
                ext().p2p_reduce(src, dst, nel, 1.0 / N, accumulate)
            ev = torch.cuda.Event()
            ev.record(self.stream)
        slot.event = None  # set when the next reduction's barrier passes
        self._prev_slot = slot
        return _P2PHandle(ev, prof)

    def wait(self, h: _P2PHandle) -> None:
        if h.torch_handle is not None:
            return self._fallback.wait(h.torch_handle)
        torch.cuda.current_stream().wait_event(h.event)
        if h.profile is not None:
            h.profile.complete()
