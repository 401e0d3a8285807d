"""Split-K policy of the weight-gradient GEMMs (a wave model with the fp32
slab cost), checked on the host for the GEMMs of one Qwen3-0.6B step
(8,192 tokens, 74 SM pairs): only o_proj's gradient (1024 x 2048 output,
32 CTA-pair tiles) splits, into two slabs; the products with enough tiles
stay unsplit, as do short-K and narrow products.  No GPU needed."""
import pytest

from parallel_b200.ops.gemm import _splitk

T = 8192


@pytest.mark.parametrize("name,M,N,want", [
    ("qkv", 4096, 1024, 1),
    ("o_proj", 1024, 2048, 2),
    ("gate_up", 6144, 1024, 1),
    ("down", 1024, 3072, 1),
    ("lm_head", 151936, 1024, 1),
])
def test_step_weight_gradients(name, M, N, want):
    assert _splitk(M, N, T, slots=74) == want, name


def test_short_k_and_narrow_products_stay_unsplit():
    assert _splitk(1024, 2048, 256, slots=74) == 1    # too few k-blocks per slice
    assert _splitk(128, 2048, 65536, slots=74) == 1   # fewer than 256 rows: one-CTA kernel
