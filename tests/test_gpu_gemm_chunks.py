"""GPU parity of the chunk-split pre-pass GEMM (b2k_gemm_set_chunk_split).

With the split, every 128 x 128 output tile is computed by one CTA per
256-wide K chunk, each storing its chunk's raw TMEM accumulator, and a second
kernel folds the chunks in order (acc = 0, then acc + chunk with
round-to-nearest per chunk) before the divisor, bias and ReLU.  That is the
unsplit kernel's own fold, so the result must be the same bits, and within
the 3xTF32 normwise bound against float64 (max|C - C64| / max|C64| <= 1e-5).
The launch counter shows which path ran: the split call launches the operand
split, the chunk kernel and the fold (three kernels), the unsplit one two.
"""
from __future__ import annotations

import numpy as np
import pytest

from oracle import tf32

pytestmark = pytest.mark.gpu

NORMWISE = 1e-5


def dev(torch, array):
    return torch.from_numpy(np.ascontiguousarray(array)).cuda()


CASES = [
    # (m, n, k, b_layout, bias, relu)
    (256, 512, 4096, 0, False, False),   # 8 tiles, 16 chunks: the case the split is for
    (513, 1000, 777, 1, True, True),     # the ragged GEMM's row shard on eight GPUs (tail chunk of 32)
    (130, 300, 1000, 0, True, False),    # ragged M and N edges
    (1, 64, 2048, 0, False, True),       # one row
    (128, 128, 257, 0, False, False),    # two chunks: 256 and a tail of one K element (padded to 32)
    (384, 260, 520, 1, False, True),
    (640, 384, 512, 0, True, False),     # two full chunks, no tail
]


def gemm(ctx, torch, chunk_mode, da, db, m, n, k, b_layout, dbias, relu, ldc=None, div=None):
    ldc = ldc or n
    dc = torch.full((m, ldc), float("nan"), dtype=torch.float32, device="cuda")
    ctx.set_gemm_chunk_split(chunk_mode)
    ctx.set_gemm_fused_split(0)  # the pre-pass kernel, the one the split applies to
    try:
        before = ctx.kernel_launches()
        if div is None:
            ctx.gemm(da.data_ptr(), db.data_ptr(), dc.data_ptr(), m, n, k, b_layout=b_layout, ldc=ldc,
                     bias=dbias.data_ptr() if dbias is not None else 0, relu=relu)
        else:
            ctx.gemm_scaled(da.data_ptr(), db.data_ptr(), dc.data_ptr(), m, n, k, b_layout=b_layout, ldc=ldc,
                            bias=dbias.data_ptr() if dbias is not None else 0, relu=relu, div_value=div)
        ctx.sync()
        launches = ctx.kernel_launches() - before
    finally:
        ctx.set_gemm_chunk_split(1)
        ctx.set_gemm_fused_split(1)
    return dc[:, :n], launches


@pytest.mark.parametrize("m,n,k,b_layout,with_bias,relu", CASES)
def test_chunk_split_equals_unsplit(ctx, torch_cuda, m, n, k, b_layout, with_bias, relu):
    torch = torch_cuda
    rng = np.random.default_rng(m * 3 + n + k)
    a = rng.uniform(-1, 1, (m, k)).astype(np.float32)
    b = rng.uniform(-1, 1, (k, n) if b_layout == 0 else (n, k)).astype(np.float32)
    bias = rng.uniform(-0.5, 0.5, n).astype(np.float32) if with_bias else None
    da, db = dev(torch, a), dev(torch, b)
    dbias = dev(torch, bias) if bias is not None else None
    plain, plain_launches = gemm(ctx, torch, 0, da, db, m, n, k, b_layout, dbias, relu)
    split, split_launches = gemm(ctx, torch, 2, da, db, m, n, k, b_layout, dbias, relu)
    assert split_launches == plain_launches + 1, (plain_launches, split_launches)
    assert torch.equal(split, plain)
    bm = b if b_layout == 0 else b.T
    exact = a.astype(np.float64) @ bm.astype(np.float64)
    if with_bias:
        exact = exact + bias
    if relu:
        exact = np.maximum(exact, 0.0)
    assert tf32.normwise_error(split.cpu().numpy(), exact) <= NORMWISE
    # the default chooser's pick gives the same bits too
    auto, _ = gemm(ctx, torch, 1, da, db, m, n, k, b_layout, dbias, relu)
    assert torch.equal(auto, plain)


def test_chunk_split_divided_product_and_unaligned_c(ctx, torch_cuda):
    """The divisor applies before the bias as in the unsplit epilogue, and a C
    whose rows are not 16-byte aligned (odd row stride) is written by the
    fold's scalar stores."""
    torch = torch_cuda
    rng = np.random.default_rng(11)
    m, n, k = 200, 333, 1500
    a = rng.uniform(-1, 1, (m, k)).astype(np.float32)
    b = rng.uniform(-1, 1, (n, k)).astype(np.float32)
    bias = rng.uniform(-0.5, 0.5, n).astype(np.float32)
    da, db, dbias = dev(torch, a), dev(torch, b), dev(torch, bias)
    for ldc in (n, n + 3):
        plain, _ = gemm(ctx, torch, 0, da, db, m, n, k, 1, dbias, True, ldc=ldc, div=3.0)
        split, launches = gemm(ctx, torch, 2, da, db, m, n, k, 1, dbias, True, ldc=ldc, div=3.0)
        assert torch.equal(split, plain), ldc
        exact = np.maximum((a.astype(np.float64) @ b.astype(np.float64).T) / 3.0 + bias, 0.0)
        assert tf32.normwise_error(split.cpu().numpy(), exact) <= NORMWISE


def test_chunk_split_default_takes_it_for_few_tiles_and_long_k(ctx, torch_cuda):
    """Under the default setting a 256 x 512 x 4096 product (8 output tiles on
    148 SMs) runs split; a 1024 x 1024 x 256 one (one chunk) does not."""
    torch = torch_cuda
    rng = np.random.default_rng(5)
    for (m, n, k), want_split in (((256, 512, 4096), True), ((1024, 1024, 256), False)):
        a = rng.uniform(-1, 1, (m, k)).astype(np.float32)
        b = rng.uniform(-1, 1, (k, n)).astype(np.float32)
        da, db = dev(torch, a), dev(torch, b)
        _, plain_launches = gemm(ctx, torch, 0, da, db, m, n, k, 0, None, False)
        _, auto_launches = gemm(ctx, torch, 1, da, db, m, n, k, 0, None, False)
        assert (auto_launches == plain_launches + 1) == want_split, (m, n, k, plain_launches, auto_launches)


def test_chunk_split_setting_is_validated(ctx):
    for mode in (0, 1, 2):
        ctx.set_gemm_chunk_split(mode)
    ctx.set_gemm_chunk_split(1)
    with pytest.raises(Exception):
        ctx.set_gemm_chunk_split(3)
