"""Host side of the grouped expert GEMM's column tiling: the width the kernel
launcher picks (``grouped_tile_n``, 256 for products wider than 128 columns)
and the weight-gradient work tables, which must tile N by the same width
(an item past the last column tile would run a whole K loop for nothing; a
missing one would leave columns unwritten).  Runs without a GPU."""
import pytest
import torch

from parallel_b200.ops._ext import ext
from parallel_b200.ops.moe import _k_work


@pytest.mark.parametrize("n,width", [(64, 128), (128, 128), (136, 256), (768, 256), (2048, 256)])
def test_tile_width_policy(n, width):
    assert int(ext().grouped_tile_n(1, n)) == width
    assert int(ext().grouped_tile_n(2, n)) == width


@pytest.mark.parametrize("E,m_group,n", [(32, 2048, 768), (4, 256, 128), (3, 200, 300)])
def test_k_work_covers_every_tile_once(E, m_group, n):
    bn = int(ext().grouped_tile_n(2, n))
    items = _k_work(E, m_group, n, torch.device("cpu")).tolist()
    want = {(e, tm, tn) for e in range(E) for tm in range(-(-m_group // 128)) for tn in range(-(-n // bn))}
    got = [(e, tm, tn) for e, tm, tn, _ in items]
    assert len(got) == len(set(got)) == len(want) and set(got) == want
    # every item's column tile starts inside the product
    assert all(tn * bn < n for _, _, tn in got)
