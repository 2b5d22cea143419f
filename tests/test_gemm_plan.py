"""Host-side GEMM planner (tile shape and split-K choice), checked without a GPU."""
import pytest

from centrifuge_b200.ops import gemm
from centrifuge_b200.ops._ext import kernels

SMS = 148


def plan(M, N, K, epi=gemm.EPI_BF16, bn=0):
    return kernels().gemm_plan(M, N, K, epi, bn, SMS)


def test_large_gemms_use_the_cta_pair():
    for M, N, K in [(8192, 8192, 8192), (16384, 11264, 2048), (16384, 32000, 2048),
                    (8192, 2048, 5632)]:
        bn, ks, pair = plan(M, N, K)
        assert pair and bn == 256 and ks == 1, (M, N, K)


def test_forced_tiles_are_respected():
    assert plan(8192, 8192, 8192, bn=128) == (128, 1, False)
    assert plan(8192, 8192, 8192, bn=256) == (256, 1, False)
    assert plan(128, 256, 64, bn=kernels().GEMM_TILE_PAIR)[2] is True


@pytest.mark.parametrize("M,N,K", [(2560, 2048, 8192), (2048, 5632, 8192)])
def test_weight_gradients_split_k_to_fill_waves(M, N, K):
    """Tile counts just above a multiple of the SM count split K (fp32-accumulate epilogue
    only); the bf16 epilogue never splits."""
    bn, ks, pair = plan(M, N, K, epi=gemm.EPI_F32_ACC)
    assert ks > 1
    assert plan(M, N, K)[1] == 1


def test_short_k_never_splits_below_16_kblocks():
    for K in (64, 512, 1024, 1984):  # fewer than 32 k-blocks of 64
        assert plan(2560, 2048, K, epi=gemm.EPI_F32_ACC)[1] == 1
