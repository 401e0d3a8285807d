"""Host model of the stream-K work split of the CTA-pair GEMM (csrc/gemm_pair.cu:
WorkIter and streamk_fixup_kernel use the same arithmetic): every (tile, k-block)
unit is computed by exactly one SM pair, every piece of a shared tile lands in
a distinct workspace slot, and the fix-up's slot rule finds exactly the pieces
that the pairs wrote, in K order."""
import pytest


def bound(c, U, nc):
    return c * U // nc


def owner(u, U, nc):
    c = u * nc // U
    while c + 1 < nc and bound(c + 1, U, nc) <= u:
        c += 1
    while c > 0 and bound(c, U, nc) > u:
        c -= 1
    return c


def items(cid, num_tiles, num_kb, nc):
    U = num_tiles * num_kb
    u0 = u = bound(cid, U, nc)
    u1 = bound(cid + 1, U, nc)
    out = []
    while u < u1:
        tile, kb0 = divmod(u, num_kb)
        kb1 = min(num_kb, kb0 + (u1 - u))
        tag = -1 if (kb0 == 0 and kb1 == num_kb) else 2 * cid + (0 if u == u0 else 1)
        out.append((tile, kb0, kb1, tag))
        u += kb1 - kb0
    return out


@pytest.mark.parametrize("num_tiles,num_kb,nc", [(32, 128, 74), (96, 128, 74), (48, 128, 74), (128, 2374, 74),
                                                 (5, 7, 11), (74, 32, 74), (100, 33, 37)])
def test_streamk_partition_and_fixup_slots(num_tiles, num_kb, nc):
    U = num_tiles * num_kb
    if U < nc:
        pytest.skip("the launcher needs at least one unit per pair")
    covered = {}
    written = {}
    for cid in range(nc):
        its = items(cid, num_tiles, num_kb, nc)
        assert len([t for t in its if t[3] >= 0]) <= 2
        for tile, kb0, kb1, tag in its:
            for kb in range(kb0, kb1):
                assert (tile, kb) not in covered
                covered[(tile, kb)] = cid
            if tag >= 0:
                assert tag not in written, "two pieces share a workspace slot"
                written[tag] = (tile, kb0, kb1)
    assert len(covered) == U
    # fix-up: the pieces of each shared tile, from the slot rule alone
    for tile in range(num_tiles):
        t0 = tile * num_kb
        c0, c1 = owner(t0, U, nc), owner(t0 + num_kb - 1, U, nc)
        if c0 == c1:
            assert all(covered[(tile, kb)] == c0 for kb in range(num_kb))
            continue
        pieces = []
        for c in range(c0, c1 + 1):
            slot = 2 * c if bound(c, U, nc) >= t0 else 2 * c + 1
            assert slot in written and written[slot][0] == tile
            pieces.append(written[slot][1:])
        # the pieces tile [0, num_kb) in K order
        assert pieces[0][0] == 0 and pieces[-1][1] == num_kb
        assert all(a[1] == b[0] for a, b in zip(pieces, pieces[1:]))
