"""The GEMM path chooser on the CPU, through b2k_gemm_plan.

b2k_gemm_plan runs the dispatch's own decision functions (split mode, tile
width, K-chunk split) on host arithmetic alone, so the paths the measured
tables describe can be checked without a GPU: the BASELINE configurations,
the multi-GPU row shards and the few-tile long-K products the chunk split is
for.  The GPU tests check that the kernels each path launches give the same
bits.
"""
from __future__ import annotations

import pytest

from conftest import pkg

SMS = 148  # B200


@pytest.fixture(scope="module")
def rt():
    return pkg("runtime")


def plan(rt, m, n, k, **kw):
    return rt.gemm_plan(SMS, m, n, k, **kw)


def test_baseline_configs(rt):
    # 4096^3, both operands TMA-readable: A split in the kernel, 192-wide tiles
    assert plan(rt, 4096, 4096, 4096) == {"split_mode": 1, "tile_width": 192, "chunk_split": False, "chunks": 16}
    # ragged: A's 777-float rows are not TMA-readable -> both operands
    # pre-split, one wave of 132 tiles of 128 x 256
    assert plan(rt, 4097, 1000, 777, b_layout=rt.B_NK) == {"split_mode": 0, "tile_width": 256,
                                                           "chunk_split": False, "chunks": 4}


@pytest.mark.parametrize("rows,mode,width", [(2048, 0, 256), (1024, 2, 128), (512, 2, 128)])
def test_gemm_row_shards(rt, rows, mode, width):
    """4096^3 split by rows over 2, 4 and 8 GPUs: the pre-pass kernel at 2048
    rows, the transposed orientation (B split in the kernel) below."""
    p = plan(rt, rows, 4096, 4096)
    assert (p["split_mode"], p["tile_width"], p["chunk_split"]) == (mode, width, False)


@pytest.mark.parametrize("rows,chunked", [(2049, False), (1025, False), (513, True), (512, True)])
def test_ragged_row_shards(rt, rows, chunked):
    """The ragged GEMM's shards take 128-wide pre-pass tiles; the 8-GPU
    shards (40 or 32 tiles over the whole K) take the K-chunk split."""
    p = plan(rt, rows, 1000, 777, b_layout=rt.B_NK)
    assert (p["split_mode"], p["tile_width"], p["chunk_split"], p["chunks"]) == (0, 128, chunked, 4)


def test_few_tiles_long_k_takes_the_chunk_split(rt):
    p = plan(rt, 256, 512, 4096)
    assert p["split_mode"] == 0 and p["chunk_split"] and p["chunks"] == 16
    # one chunk: nothing to split
    assert not plan(rt, 256, 512, 256)["chunk_split"]


def test_chunk_setting_and_alignment_steer_the_plan(rt):
    lib = rt.library()
    try:
        assert lib.b2k_gemm_set_chunk_split(0) == rt.B2K_OK
        assert not plan(rt, 513, 1000, 777, b_layout=rt.B_NK)["chunk_split"]
        assert lib.b2k_gemm_set_chunk_split(2) == rt.B2K_OK
        assert plan(rt, 4097, 1000, 777, b_layout=rt.B_NK)["chunk_split"]
    finally:
        lib.b2k_gemm_set_chunk_split(1)
    # an A that TMA cannot read (not 16-byte aligned) cannot be split in the kernel
    assert plan(rt, 4096, 4096, 4096, a=256 + 4)["split_mode"] != 1


@pytest.mark.parametrize("args", [(0, 16, 16), (16, 0, 16), (16, 16, 0), (-1, 16, 16)])
def test_plan_refuses_what_the_gemm_refuses(rt, args):
    with pytest.raises(rt.B2KError):
        plan(rt, *args)
    with pytest.raises(rt.B2KError):
        rt.gemm_plan(0, 16, 16, 16)  # no SMs
    with pytest.raises(rt.B2KError):
        plan(rt, 16, 16, 16, lda=8)  # leading dimension shorter than K
