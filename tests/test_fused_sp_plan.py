"""Address plans of the pull mode of the sequence-parallel collectives
(``pull_gather_plan`` / ``pull_reduce_plan``), executed on host memory by an
emulation of the peer copy and N-peer reduce kernels: every rank's buffer is
a slice of one byte arena, pointers are arena addresses."""
import pytest
import torch

from parallel_b200.parallel.model_parallel.fused_sp import pull_gather_plan, pull_reduce_plan


class Arena:
    def __init__(self, nbytes):
        self.raw = torch.zeros(nbytes, dtype=torch.uint8)
        self.base = self.raw.data_ptr()
        self.top = 0

    def alloc(self, shape, dtype=torch.bfloat16):
        n = torch.Size(shape).numel() * torch.empty(0, dtype=dtype).element_size()
        t = self.raw[self.top:self.top + n].view(dtype).view(shape)
        self.top += (n + 255) // 256 * 256
        return t

    def _bytes(self, ptr, n):
        off = ptr - self.base
        assert 0 <= off and off + n <= self.raw.numel()
        return self.raw[off:off + n]

    def copy(self, src, dst, nbytes):
        for s, d, n in zip(src, dst, nbytes):
            self._bytes(d, n).copy_(self._bytes(s, n))

    def reduce(self, src, dst, nelem, scale, accumulate):
        for i, (d, n) in enumerate(zip(dst, nelem)):
            acc = sum(self._bytes(peer[i], 2 * n).view(torch.bfloat16).float() for peer in src) * scale
            out = self._bytes(d, 2 * n).view(torch.bfloat16)
            out.copy_((out.float() + acc) if accumulate else acc)


@pytest.mark.parametrize("world,batch,seq", [(2, 1, 8), (4, 2, 16), (8, 3, 32)])
def test_pull_gather_assembles_every_sequence_in_position_order(world, batch, seq):
    cols, sl = 8, seq // world
    A = Arena(1 << 20)
    shards = [A.alloc((batch * sl, cols)) for _ in range(world)]
    for j, s in enumerate(shards):
        s.copy_(torch.arange(s.numel(), dtype=torch.float32).view_as(s) + 1000 * j)
    for rank in range(world):
        full = A.alloc((batch * seq, cols))
        ptrs = [s.data_ptr() for s in shards]
        src, dst, nbytes = pull_gather_plan(ptrs, full.data_ptr(), batch, seq, cols, rank=rank)
        assert all(x % 16 == 0 for x in src + dst + nbytes)   # the copy kernel's alignment rule
        # the rank reads its own shard first, then rank+1, ...: ranks start on different sources
        assert src[0] == ptrs[rank] and src[batch] == ptrs[(rank + 1) % world]
        A.copy(src, dst, nbytes)
        want = torch.cat([torch.cat([shards[j][b * sl:(b + 1) * sl] for j in range(world)]) for b in range(batch)])
        assert torch.equal(full, want)


@pytest.mark.parametrize("world,batch,seq", [(2, 1, 8), (4, 2, 16), (8, 3, 32)])
def test_pull_reduce_sums_each_owners_rows_from_every_peer(world, batch, seq):
    cols, sl = 8, seq // world
    A = Arena(1 << 21)
    g = torch.Generator().manual_seed(0)
    parts = [A.alloc((batch * seq, cols)) for _ in range(world)]
    for p in parts:
        p.copy_(torch.randint(-8, 8, p.shape, generator=g).float())
    total = sum(p.float() for p in parts).view(batch, seq, cols)
    for rank in range(world):
        y = A.alloc((batch * sl, cols))
        src, dst, nelem = pull_reduce_plan([p.data_ptr() for p in parts], y.data_ptr(), rank, batch, seq, cols)
        assert all(s % 16 == 0 for peer in src for s in peer) and all(d % 16 == 0 for d in dst)
        assert all(n % 8 == 0 for n in nelem)
        A.reduce(src, dst, nelem, 1.0, False)
        want = total[:, rank * sl:(rank + 1) * sl].reshape(batch * sl, cols)
        assert torch.equal(y.float(), want)
