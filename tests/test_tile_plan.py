"""The tensor-core tile and split-K choice, as pure host logic (gs_plan_tile), against the decisions the
timed sweep of every tile backs (the tile-choice and split-K profiles): the north-star configurations keep
the wide 256x512 tile; one round of 1-SM tiles takes the 1-SM tile; small batched problems take the pair
tile; calls of at most 4 K stages take the wide tile; long-K single GEMMs with few tiles split K."""
import pytest

import gemm_sm100 as gs

F16, BF16, I8, F32, I32 = gs.R_16F, gs.R_16BF, gs.R_8I, gs.R_32F, gs.R_32I
C32F, C32I = gs.COMPUTE_32F, gs.COMPUTE_32I


def plan(m, n, k, batch=1, at=F16, ct=F32, comp=C32F, algo=gs.GEMM_DEFAULT, ta=0, tb=0, sms=148):
    st, tile, parts = gs.plan_tile(ta, tb, m, n, k, at, ct, comp, batch=batch, algo=algo, sm_count=sms)
    assert st == gs.STATUS_SUCCESS
    return tile, parts


@pytest.mark.parametrize("m,n,k,batch,at,ct,comp", [
    (8192, 8192, 8192, 1, F16, F32, C32F),      # C3
    (8192, 8192, 8192, 1, BF16, F32, C32F),     # C3 bf16
    (4096, 4096, 4096, 1, F16, F32, C32F),      # C3 4096^3
    (8192, 8192, 8192, 1, I8, I32, C32I),       # C5
    (512, 512, 1024, 256, F16, F32, C32F),      # C4
    (2048, 2048, 2048, 64, I8, I32, C32I),      # C5b
])
def test_north_star_configurations_keep_the_wide_tile(m, n, k, batch, at, ct, comp):
    assert plan(m, n, k, batch, at, ct, comp) == (gs.TILE_WIDE, 1)


@pytest.mark.parametrize("m,n,k", [(1024, 1024, 1024), (2048, 2048, 2048), (1536, 1536, 1536), (1024, 4096, 2048)])
def test_one_round_of_1sm_tiles_takes_the_1sm_tile(m, n, k):
    assert plan(m, n, k) == (gs.TILE_1SM, 1)
    assert plan(m, n, k, at=I8, ct=I32, comp=C32I) == (gs.TILE_1SM, 1)


@pytest.mark.parametrize("m,n,k,batch", [(768, 768, 768, 64), (1024, 1024, 1024, 32), (1280, 1280, 1280, 8)])
def test_small_batched_problems_take_the_pair_tile(m, n, k, batch):
    assert plan(m, n, k, batch) == (gs.TILE_PAIR, 1)


@pytest.mark.parametrize("m,n,k,batch", [(512, 512, 512, 64), (512, 512, 768, 64), (512, 1024, 512, 96)])
def test_16bit_short_k_batches_take_the_pair_tile(m, n, k, batch):
    """5-15 K stages of 16-bit operands: the wide tile's exposed drain tips these to the pair tile."""
    assert plan(m, n, k, batch) == (gs.TILE_PAIR, 1)
    assert plan(m, n, k, batch, at=BF16, ct=BF16)[0] == gs.TILE_PAIR


def test_short_k_takes_the_wide_tile():
    assert plan(8192, 4096, 256, at=I8, ct=I32, comp=C32I) == (gs.TILE_WIDE, 1)
    assert plan(1024, 1024, 256, 64, at=I8, ct=I32, comp=C32I) == (gs.TILE_WIDE, 1)


def test_m_at_most_128_takes_the_1sm_tile():
    assert plan(128, 4096, 4096)[0] == gs.TILE_1SM
    assert plan(64, 8192, 512, 16)[0] == gs.TILE_1SM


@pytest.mark.parametrize("algo,tile", [(0, gs.TILE_1SM), (1, gs.TILE_PAIR), (2, gs.TILE_WIDE)])
def test_algo_hint_forces_the_tile_and_keeps_one_launch(algo, tile):
    assert plan(8192, 8192, 8192, algo=algo) == (tile, 1)
    assert plan(512, 512, 16384, algo=algo) == (tile, 1)


def test_long_k_with_few_tiles_splits_k():
    assert plan(512, 512, 16384) == (gs.TILE_PAIR, 16)
    assert plan(512, 512, 16384, at=I8, ct=I32, comp=C32I) == (gs.TILE_PAIR, 8)
    assert plan(1024, 1024, 4096) == (gs.TILE_PAIR, 4)
    assert plan(256, 1024, 32768) == (gs.TILE_PAIR, 16)
    # every slice keeps at least 16 stages of 64 K elements (f16)
    for k in (2048, 4096, 8192, 16384, 32768):
        tile, parts = plan(512, 512, k)
        assert parts == 1 or (k // parts) >= 16 * 64


def test_split_k_is_not_taken():
    assert plan(512, 512, 16384 + 8)[1] == 1        # K not a whole number of stages
    assert plan(512, 512, 16384, batch=2)[1] == 1   # batched calls
    assert plan(4096, 4096, 16384)[1] == 1          # enough tiles to fill the GPU
    assert plan(1024, 1024, 1024)[1] == 1           # too few K stages per slice
    assert plan(1024, 1024, 4096, at=I8, ct=I32, comp=C32I)[1] == 1  # two slices would not pay for the reduction


def test_smaller_gpu_scales_the_rounds():
    # with a quarter of the SMs, 2048^3 is no longer one round of 1-SM tiles
    assert plan(2048, 2048, 2048, sms=148)[0] == gs.TILE_1SM
    assert plan(2048, 2048, 2048, sms=36)[0] != gs.TILE_1SM


def test_fp32_and_bad_arguments():
    st, tile, parts = gs.plan_tile(0, 0, 512, 512, 512, F32, F32, C32F)
    assert st == gs.STATUS_NOT_SUPPORTED
    st, _, _ = gs.plan_tile(0, 0, -1, 512, 512, F16, F32, C32F)
    assert st == gs.STATUS_INVALID_VALUE
    st, tile, parts = gs.plan_tile(0, 0, 0, 512, 512, F16, F32, C32F)
    assert st == gs.STATUS_SUCCESS and tile == 0
