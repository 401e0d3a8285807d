"""Tensor- and sequence-parallel collectives fused with their GEMMs over NVLink.

Megatron-style sequence parallelism surrounds every column-parallel GEMM with
an all-gather of the sequence-sharded activations and every row-parallel GEMM
with a reduce-scatter of its partial output (the reference issues both through
NCCL around HF's Linear layers: parallel/parallel/engine/model_parallel/
sequence_parallel.py:19-46,178-213, tensor_parallel.py:31-35).  Here each pair
is one kernel (``csrc/gemm_pair.cu``):

* all-gather -> GEMM (``gemm_ag``): every rank's shard sits in a symmetric
  buffer; copy warps inside the GEMM kernel pull the peers' shards over
  NVLink into a local gathered buffer one 256-row block at a time and publish
  per-block counters, and the GEMM starts each tile as soon as its block is
  in (local shard first, then the peers in rotation).  The gathered buffer is
  kept for the weight gradient.
* GEMM -> reduce-scatter (``gemm_rs``): the epilogue stores every output row
  of the partial product straight into its owner's symmetric receive buffer
  (one slot per sender); after a signal barrier the owner sums its slots.

Buffers rotate between two sets, so one signal barrier per call orders reuse:
when a rank passes the barrier of call k every rank has finished call k-1,
hence nobody still reads the set that call k+1 overwrites.

``mode="pull"`` (the default; ``PB_SP_MODE=fused`` selects the in-GEMM
variant above) runs the same two operations as a
collective followed / preceded by a plain GEMM, with no communication inside
the GEMM kernel: the all-gather is one peer-gather kernel (every rank pulls
the peers' shards into the gathered buffer), the reduce-scatter writes the
whole partial product into this rank's symmetric buffer with the GEMM's
TMA-store epilogue and each owner then pulls and sums its rows from every
peer with the N-peer reduce kernel.  It trades the overlap of the fused
kernels for bulk transfers (no per-row peer stores from the epilogue); the
address plans are ``pull_gather_plan`` / ``pull_reduce_plan``.
"""
from __future__ import annotations

import os

import torch
import torch.distributed as dist

from ...ops._ext import ext
from ...ops.gemm import EPI_STORE_BF16, EPI_SWIGLU
from ...profiling import collective_profile
from ..comm.p2p import NvlsAllReduce, SymmBuffer, p2p_supported

_PIECES_PER_BLOCK = 256 // 16  # kGatherRowsPerPiece = 16 rows per copy piece


def pull_gather_plan(peer_ptrs: list[int], dst_ptr: int, batch: int, seq: int, cols: int, es: int = 2,
                     rank: int = 0):
    """Peer-gather arguments (src, dst, nbytes) that assemble the gathered
    [batch*seq, cols] activation from every rank's [batch*seq/world, cols]
    shard: rank j holds positions [j*sl, (j+1)*sl) of every sequence.  The
    segments start at ``rank``'s own shard and walk the peers from rank+1, so
    the ranks of a group read different sources at any moment."""
    world = len(peer_ptrs)
    sl = seq // world
    seg = sl * cols * es
    src, dst = [], []
    for i in range(world):
        j = (rank + i) % world
        p = peer_ptrs[j]
        for b in range(batch):
            src.append(p + b * seg)
            dst.append(dst_ptr + (b * seq + j * sl) * cols * es)
    return src, dst, [seg] * len(src)


def pull_reduce_plan(peer_ptrs: list[int], dst_ptr: int, rank: int, batch: int, seq: int, cols: int, es: int = 2):
    """N-peer reduce arguments (src per peer, dst, nelem) that sum this rank's
    rows - positions [rank*sl, (rank+1)*sl) of every sequence - out of every
    peer's full [batch*seq, cols] partial product into the local
    [batch*seq/world, cols] output."""
    world = len(peer_ptrs)
    sl = seq // world
    rows = [(b * seq + rank * sl) * cols * es for b in range(batch)]
    src = [[p + r for r in rows] for p in peer_ptrs]
    dst = [dst_ptr + b * sl * cols * es for b in range(batch)]
    return src, dst, [sl * cols] * batch


class FusedSequenceParallel:
    """NVLink data plane of one TP/SP group (all ranks call in the same order)."""

    def __init__(self, group, device: torch.device, mode: str | None = None):
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        self.device = device
        # pull (default): peer-gather kernel + GEMM, GEMM + owner-pull reduce;
        # measured faster than the in-GEMM variant at 4 GPUs (GEMM -> reduce-
        # scatter 1.09x vs 0.66x of NCCL + cuBLAS, all-gather -> GEMM 0.91x vs 0.85x)
        self.mode = mode or os.environ.get("PB_SP_MODE", "pull")
        if self.mode not in ("fused", "pull"):
            raise ValueError(f"unknown sequence-parallel mode {self.mode!r} (fused / pull)")
        self.limit_s = float(os.environ.get("PB_P2P_TIMEOUT_S", "60"))
        self._rows = 0
        self._cols = 0
        self.ag = []  # 2 x SymmBuffer [rows_local, cols] (this rank's shard)
        self.rs = []  # 2 x SymmBuffer [world * rows_local, cols] (one slot per sender)
        self.flags = []
        self.n_ag = 0
        self.n_rs = 0

    # ------------------------------------------------------------------ support
    @staticmethod
    def available(group, device) -> bool:
        return device.type == "cuda" and p2p_supported(group)

    def supports(self, batch: int, seq: int, cols: int) -> bool:
        """Shapes the fused kernels take: 256-row aligned local shards, <= 64 row blocks."""
        if seq % self.world:
            return False
        sl = seq // self.world
        return sl % 256 == 0 and (batch * seq) // 256 <= 64 and cols % 8 == 0

    def _ensure(self, rows_local: int, cols: int) -> None:
        if self.ag and rows_local <= self._rows and cols <= self._cols:
            return
        if self.ag:
            raise RuntimeError("fused sequence parallel: buffers are sized by the first call; shapes grew "
                               f"({self._rows}x{self._cols} -> {rows_local}x{cols})")
        self._rows, self._cols = rows_local, cols
        n = rows_local * cols
        self.ag = [SymmBuffer(n, torch.bfloat16, self.device, self.group, "sp_gather") for _ in range(2)]
        self.rs = [SymmBuffer(self.world * n, torch.bfloat16, self.device, self.group, "tp_partials")
                   for _ in range(2)]
        self.flags = [torch.zeros(64, dtype=torch.int32, device=self.device) for _ in range(2)]

    def _block_order(self, batch: int, seq: int) -> list[int]:
        sl = seq // self.world
        blocks = list(range(batch * seq // 256))
        owner = [((b * 256) % seq) // sl for b in blocks]
        return sorted(blocks, key=lambda b: ((owner[b] - self.rank) % self.world, b))

    # ------------------------------------------------------------------ all-gather -> GEMM
    def all_gather_gemm(self, x_local: torch.Tensor, b: torch.Tensor, batch: int, seq: int, *, b_mn: bool = False,
                        swiglu_inter: int = 0, gu_out: torch.Tensor | None = None):
        """Returns (out, x_full): out = gather(x) @ b^T (or @ b when b_mn), or for
        swiglu_inter > 0 the SwiGLU of the gate/up product (gu_out receives the
        pre-activations); x_full [batch*seq, K] is the gathered input."""
        rows_local, K = x_local.shape
        self._ensure(rows_local, K)
        k = self.n_ag % 2
        buf = self.ag[k]
        shard = buf.tensor[: rows_local * K].view(rows_local, K)
        shard.copy_(x_local)
        T = batch * seq
        x_full = torch.empty(T, K, device=x_local.device, dtype=torch.bfloat16)
        if swiglu_inter:
            out = torch.empty(T, swiglu_inter, device=x_local.device, dtype=torch.bfloat16)
            epi, n_out, up = EPI_SWIGLU, swiglu_inter, swiglu_inter
        else:
            N = b.shape[1] if b_mn else b.shape[0]
            out = torch.empty(T, N, device=x_local.device, dtype=torch.bfloat16)
            epi, n_out, up = EPI_STORE_BF16, 0, 0
        n_cols = 2 * swiglu_inter if swiglu_inter else out.shape[1]
        if self.mode == "pull":
            with collective_profile("sp_all_gather_gemm", value=x_local, mode="pull", flops=2.0 * T * K * n_cols,
                                    link_bytes=(self.world - 1) * rows_local * K * 2):
                buf.barrier(0, self.limit_s)
                ext().p2p_copy(*pull_gather_plan(buf.peer_ptrs, x_full.data_ptr(), batch, seq, K, rank=self.rank))
                if swiglu_inter:
                    ext().gemm(x_full, b, out, False, False, EPI_SWIGLU, 1.0, gu_out, up, n_out)
                else:
                    ext().gemm(x_full, b, out, False, b_mn, EPI_STORE_BF16, 1.0)
            self.n_ag += 1
            return out, x_full
        # per-call block counters: zeroed on the stream, so the target is a
        # constant and a captured CUDA graph replays the same launch
        self.flags[k].zero_()
        target = _PIECES_PER_BLOCK
        with collective_profile("sp_all_gather_gemm", value=x_local, mode="fused", flops=2.0 * T * K * n_cols,
                                link_bytes=(self.world - 1) * rows_local * K * 2):
            buf.barrier(0, self.limit_s)
            ext().gemm_ag(x_full, buf.peer_ptrs, K, self.flags[k], target, seq, seq // self.world, batch,
                          self._block_order(batch, seq), b, out, b_mn, epi, 1.0, gu_out, up, n_out)
        self.n_ag += 1
        return out, x_full

    # ------------------------------------------------------------------ GEMM -> reduce-scatter
    def gemm_reduce_scatter(self, a_full: torch.Tensor, b: torch.Tensor, batch: int, seq: int, *,
                            b_mn: bool = False) -> torch.Tensor:
        """y_local [batch*seq/world, N] = reduce_scatter(a_full @ b^T (or @ b))."""
        N = b.shape[1] if b_mn else b.shape[0]
        rows_local = batch * seq // self.world
        self._ensure(rows_local, N)  # receive slots are rows_local x N (N <= buffer width)
        k = self.n_rs % 2
        buf = self.rs[k]
        y = torch.empty(rows_local, N, device=a_full.device, dtype=torch.bfloat16)
        slot_elems = rows_local * N
        if self.mode == "pull":
            T = a_full.shape[0]
            part = buf.tensor[: T * N].view(T, N)
            with collective_profile("sp_gemm_reduce_scatter", payload_bytes=T * N * 2, mode="pull",
                                    flops=2.0 * T * a_full.shape[1] * N,
                                    link_bytes=(self.world - 1) * rows_local * N * 2):
                ext().gemm(a_full, b, part, False, b_mn, EPI_STORE_BF16, 1.0)
                buf.barrier(0, self.limit_s)
                ext().p2p_reduce(*pull_reduce_plan(buf.peer_ptrs, y.data_ptr(), self.rank, batch, seq, N), 1.0,
                                 False)
            self.n_rs += 1
            return y
        with collective_profile("sp_gemm_reduce_scatter", payload_bytes=a_full.shape[0] * N * 2, mode="fused",
                                flops=2.0 * a_full.shape[0] * a_full.shape[1] * N,
                                link_bytes=(self.world - 1) * rows_local * N * 2):
            ext().gemm_rs(a_full, b, b_mn, 1.0, buf.peer_ptrs, N, seq, seq // self.world, self.rank, rows_local)
            buf.barrier(0, self.limit_s)
            base = buf.tensor.data_ptr()
            ext().p2p_reduce([[base + s * slot_elems * 2] for s in range(self.world)], [y.data_ptr()],
                             [slot_elems], 1.0, False)
        self.n_rs += 1
        return y


class FusedTensorParallel:
    """The same data-plane interface for tensor parallelism WITHOUT sequence
    parallelism, so the fused autograd Functions below serve both modes.  The
    reference's non-SP TP all-reduces the row-parallel outputs in forward and
    the column-parallel input gradients in backward (HF Rowwise / Colwise
    styles, hf/integrations/tensor_parallel.py:702,845).  Here:

    * ``all_gather_gemm``: the input is replicated, so the "gather" is the
      identity and this is a plain GEMM (optionally with the SwiGLU epilogue);
    * ``gemm_reduce_scatter`` is a GEMM -> all-reduce: the GEMM epilogue stores
      every row of the partial product into its row owner's symmetric slot
      over NVLink (the reduce-scatter's transfer rides inside the GEMM), the
      owner sums its slots into a symmetric block, and every rank gathers the
      reduced blocks of all owners.  Two signal barriers; buffers rotate over
      two sets (a rank passing call k's barriers knows every rank finished
      call k-1, so the set call k+1 overwrites is free)."""

    def __init__(self, group, device: torch.device):
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        self.device = device
        self.limit_s = float(os.environ.get("PB_P2P_TIMEOUT_S", "60"))
        self._rows = 0
        self._cols = 0
        self.rs = []   # 2 x SymmBuffer [world * rows_local, cols]: one receive slot per sender
        self.red = []  # 2 x SymmBuffer [rows_local, cols]: this rank's reduced row block
        self.n = 0

    available = staticmethod(FusedSequenceParallel.available)

    def supports(self, batch: int, seq: int, cols: int) -> bool:
        rows = batch * seq
        if rows % self.world or cols % 8:
            return False
        return not self.rs or (rows // self.world <= self._rows and cols <= self._cols)

    def _ensure(self, rows_local: int, cols: int) -> None:
        if self.rs and rows_local <= self._rows and cols <= self._cols:
            return
        if self.rs:
            raise RuntimeError("fused tensor parallel: buffers are sized by the first call; shapes grew "
                               f"({self._rows}x{self._cols} -> {rows_local}x{cols})")
        self._rows, self._cols = rows_local, cols
        n = rows_local * cols
        self.rs = [SymmBuffer(self.world * n, torch.bfloat16, self.device, self.group, "tp_partials")
                   for _ in range(2)]
        self.red = [SymmBuffer(n, torch.bfloat16, self.device, self.group, "tp_reduced") for _ in range(2)]

    def all_gather_gemm(self, x: torch.Tensor, b: torch.Tensor, batch: int, seq: int, *, b_mn: bool = False,
                        swiglu_inter: int = 0, gu_out: torch.Tensor | None = None):
        T = x.shape[0]
        if swiglu_inter:
            out = torch.empty(T, swiglu_inter, device=x.device, dtype=torch.bfloat16)
            ext().gemm(x, b, out, False, False, EPI_SWIGLU, 1.0, gu_out, swiglu_inter, swiglu_inter)
        else:
            N = b.shape[1] if b_mn else b.shape[0]
            out = torch.empty(T, N, device=x.device, dtype=torch.bfloat16)
            ext().gemm(x, b, out, False, b_mn, EPI_STORE_BF16, 1.0)
        return out, x

    def _order(self) -> list[int]:
        """Peer order of this rank's copies: itself first, then rank+1, ...
        (a common order would send every rank to the same peer at once)."""
        return [(self.rank + i) % self.world for i in range(self.world)]

    def _reduce_and_gather(self, rs, red, y: torch.Tensor, slot: int) -> None:
        rs.barrier(0, self.limit_s)
        base = rs.tensor.data_ptr()
        ext().p2p_reduce([[base + s * slot * 2] for s in range(self.world)], [red.tensor.data_ptr()], [slot],
                         1.0, False)
        red.barrier(0, self.limit_s)
        order = self._order()
        ext().p2p_copy([red.peer_ptrs[r] for r in order], [y.data_ptr() + r * slot * 2 for r in order],
                       [slot * 2] * self.world)

    def try_all_reduce(self, x: torch.Tensor):
        """SUM of a bf16 CUDA tensor over the group: through the switch
        (``NvlsAllReduce``) where the group has NVLS, else on the same buffers
        as the sequence-parallel collectives (row blocks pushed to their
        owners, owner reduce, gather).  None when the shape does not fit
        (rows % world, or larger than the buffers sized by the first call), so
        the caller falls back to NCCL."""
        if not (x.is_cuda and x.dtype == torch.bfloat16 and x.dim() >= 1 and x.shape[-1] % 8 == 0):
            return None
        x2 = x.reshape(-1, x.shape[-1]).contiguous()
        M, N = x2.shape
        nv = NvlsAllReduce.get(self.group, x.device, M * N)
        if nv is not None and x2.data_ptr() % 16 == 0:
            y = torch.empty(M, N, device=x.device, dtype=torch.bfloat16)
            with collective_profile("tp_all_reduce", value=x2, mode="nvls"):
                nv.all_reduce_([x2], 1.0, outs=[y])
            return y.view(x.shape)
        if M % self.world:
            return None
        rows_local = M // self.world
        if self.rs and (rows_local > self._rows or N > self._cols):
            return None
        self._ensure(rows_local, N)
        x2 = x2.contiguous()
        k = self.n % 2
        rs, red = self.rs[k], self.red[k]
        slot = rows_local * N
        y = torch.empty(M, N, device=x.device, dtype=torch.bfloat16)
        with collective_profile("tp_all_reduce", value=x2, mode="p2p"):
            order = self._order()
            ext().p2p_copy([x2.data_ptr() + r * slot * 2 for r in order],
                           [rs.peer_ptrs[r] + self.rank * slot * 2 for r in order], [slot * 2] * self.world)
            self._reduce_and_gather(rs, red, y, slot)
        self.n += 1
        return y.view(x.shape)

    def gemm_reduce_scatter(self, a: torch.Tensor, b: torch.Tensor, batch: int, seq: int, *,
                            b_mn: bool = False) -> torch.Tensor:
        """y [M, N] = all_reduce(a @ b^T (or @ b)) over the group (see the class docstring)."""
        M = a.shape[0]
        N = b.shape[1] if b_mn else b.shape[0]
        rows_local = M // self.world
        self._ensure(rows_local, N)
        k = self.n % 2
        rs, red = self.rs[k], self.red[k]
        slot = rows_local * N
        y = torch.empty(M, N, device=a.device, dtype=torch.bfloat16)
        with collective_profile("tp_gemm_all_reduce", payload_bytes=M * N * 2, mode="fused",
                                flops=2.0 * M * a.shape[1] * N, link_bytes=2 * (self.world - 1) * slot * 2):
            ext().gemm_rs(a, b, b_mn, 1.0, rs.peer_ptrs, N, M, rows_local, self.rank, rows_local)
            self._reduce_and_gather(rs, red, y, slot)
        self.n += 1
        return y


# ---------------------------------------------------------------------------- autograd
class _LinearRSFn(torch.autograd.Function):
    """Row-parallel linear with the sequence reduce-scatter fused (forward) and
    the all-gather of the output gradient fused into the dgrad GEMM (backward)."""

    @staticmethod
    def forward(ctx, a, w, sp, batch, seq):
        a2 = a.reshape(-1, a.shape[-1])
        if not a2.is_contiguous():
            a2 = a2.contiguous()
        y = sp.gemm_reduce_scatter(a2, w, batch, seq)
        ctx.save_for_backward(a2, w)
        ctx.sp, ctx.batch, ctx.seq = sp, batch, seq
        return y

    @staticmethod
    def backward(ctx, g):
        from ...ops import gemm as G

        a2, w = ctx.saved_tensors
        g2 = g.reshape(-1, w.shape[0])
        if not g2.is_contiguous():
            g2 = g2.contiguous()
        da, g_full = ctx.sp.all_gather_gemm(g2, w, ctx.batch, ctx.seq, b_mn=True)
        dw = G.linear_wgrad(g_full, a2)
        return da, dw, None, None, None


def linear_reduce_scatter(a, w, sp: FusedSequenceParallel, batch: int, seq: int):
    """reduce_scatter_seq(a @ w.T) -> [batch*seq/world, out]."""
    return _LinearRSFn.apply(a, w, sp, batch, seq)


class _SPMLPFn(torch.autograd.Function):
    """Dense SwiGLU MLP under sequence parallelism: gather -> gate/up (SwiGLU
    epilogue) in one kernel, down -> reduce-scatter in one kernel; the backward
    mirrors it (gather of dy fused into the down dgrad, reduce-scatter of dx
    fused into the gate/up dgrad)."""

    @staticmethod
    def forward(ctx, x_local, wg, wu, wd, sp, batch, seq):
        from ...ops.functional import fused_rows

        I = wg.shape[0]
        x2 = x_local.reshape(-1, x_local.shape[-1])
        if not x2.is_contiguous():
            x2 = x2.contiguous()
        wgu = fused_rows(wg, wu)
        T = batch * seq
        gu = torch.empty(T, 2 * I, device=x2.device, dtype=torch.bfloat16)
        h, x_full = sp.all_gather_gemm(x2, wgu, batch, seq, swiglu_inter=I, gu_out=gu)
        y = sp.gemm_reduce_scatter(h, wd, batch, seq)
        ctx.save_for_backward(x_full, wg, wu, wd, gu, h)
        ctx.sp, ctx.batch, ctx.seq = sp, batch, seq
        ctx.in_shape = x_local.shape
        return y.view(*x_local.shape[:-1], wd.shape[0])

    @staticmethod
    def backward(ctx, dy):
        from ...ops import gemm as G
        from ...ops.functional import fused_rows

        x_full, wg, wu, wd, gu, h = ctx.saved_tensors
        I = wg.shape[0]
        dy2 = dy.reshape(-1, wd.shape[0])
        if not dy2.is_contiguous():
            dy2 = dy2.contiguous()
        dh, dy_full = ctx.sp.all_gather_gemm(dy2, wd, ctx.batch, ctx.seq, b_mn=True)
        dwd = G.linear_wgrad(dy_full, h)
        dgu = torch.empty_like(gu)
        ext().swiglu_bwd(dh, gu, dgu)
        wgu = fused_rows(wg, wu)
        dx = ctx.sp.gemm_reduce_scatter(dgu, wgu, ctx.batch, ctx.seq, b_mn=True).view(ctx.in_shape)
        dwgu = G.linear_wgrad(dgu, x_full)
        return dx, dwgu[:I], dwgu[I:], dwd, None, None, None


def sp_swiglu_mlp(x_local, wg, wu, wd, sp: FusedSequenceParallel, batch: int, seq: int):
    return _SPMLPFn.apply(x_local, wg, wu, wd, sp, batch, seq)
