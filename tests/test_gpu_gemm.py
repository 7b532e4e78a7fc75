"""GPU parity of the tcgen05 3xTF32 GEMM through the C ABI.

Tolerances: the matmul family's metadata tolerance (rtol = atol = 1e-3,
tools/research_cases.py:30-35) elementwise against the float64 reference, and
the north-star bound for 3xTF32 evaluated normwise:
max|C - C64| / max|C64| <= 1e-5.
"""
from __future__ import annotations

import numpy as np
import pytest

from conftest import pkg
from oracle import refs, tf32

pytestmark = pytest.mark.gpu

NORMWISE = 1e-5


def dev(torch, array):
    return torch.from_numpy(np.ascontiguousarray(array)).cuda()


def run_gemm(ctx, torch, a, b, *, b_layout=0, bias=None, relu=False):
    m, k = a.shape
    n = b.shape[1] if b_layout == 0 else b.shape[0]
    da, db = dev(torch, a), dev(torch, b)
    dc = torch.full((m, n), float("nan"), dtype=torch.float32, device="cuda")
    dbias = dev(torch, bias) if bias is not None else None
    ctx.gemm(da.data_ptr(), db.data_ptr(), dc.data_ptr(), m, n, k, b_layout=b_layout,
             bias=dbias.data_ptr() if dbias is not None else 0, relu=relu)
    ctx.sync()
    return dc.cpu().numpy()


@pytest.mark.parametrize("m,n,k", [(128, 256, 32), (128, 256, 64), (256, 512, 128), (512, 512, 512),
                                   (64, 65, 32), (3, 16, 31), (130, 300, 200), (1000, 257, 96)])
def test_gemm_kn_matches_float64(ctx, torch_cuda, m, n, k):
    rng = np.random.default_rng(m * 7 + n * 13 + k)
    a = rng.uniform(-1, 1, (m, k)).astype(np.float32)
    b = rng.uniform(-1, 1, (k, n)).astype(np.float32)
    got = run_gemm(ctx, torch_cuda, a, b)
    exact = a.astype(np.float64) @ b.astype(np.float64)
    assert tf32.normwise_error(got, exact) <= NORMWISE
    ok, bad, err = refs.allclose_report(got, refs.matmul(a, b), 1e-3, 1e-3)
    assert ok, (bad, err)


def test_gemm_matches_3xtf32_model(ctx, torch_cuda):
    """Against the oracle's 3xTF32 contract (hh + hl + lh, lo*lo dropped)."""
    rng = np.random.default_rng(3)
    a = (rng.standard_normal((256, 384)) * 8).astype(np.float32)
    b = (rng.standard_normal((384, 256)) * 8).astype(np.float32)
    got = run_gemm(ctx, torch_cuda, a, b)
    model = tf32.gemm_3xtf32(a, b)
    exact = a.astype(np.float64) @ b.astype(np.float64)
    assert tf32.normwise_error(got, model) <= 2e-6
    assert tf32.normwise_error(got, exact) <= NORMWISE


def test_gemm_nk_bias_relu_ragged(ctx, torch_cuda):
    """The ragged configuration: M=4097, N=1000, K=777, B stored N x K, bias + ReLU."""
    workloads = pkg("workloads")
    a, bt, bias = workloads.ragged_inputs()
    got = run_gemm(ctx, torch_cuda, a, bt, b_layout=1, bias=bias, relu=True)
    expect = refs.matmul_bias_relu(a, bt, bias)
    ok, bad, err = refs.allclose_report(got, expect, 1e-3, 1e-3)
    assert ok, (bad, err)
    exact = np.maximum(a.astype(np.float64) @ bt.astype(np.float64).T + bias, 0.0)
    assert tf32.normwise_error(got, exact) <= NORMWISE


def test_gemm_maxfinite_times_zero(ctx, torch_cuda):
    """The bundled TF32 range witness: lhs max-finite, rhs zeros, expected 0."""
    a = np.full((16, 8), np.finfo(np.float32).max, dtype=np.float32)
    b = np.zeros((8, 8), dtype=np.float32)
    got = run_gemm(ctx, torch_cuda, a, b)
    np.testing.assert_array_equal(got, np.zeros((16, 8), np.float32))


def test_gemm_4096_cubed(ctx, torch_cuda):
    """The benchmark configuration: every one of the 4096 x 4096 outputs
    against float64 (the host BLAS does the whole product in well under a
    second), normwise and at the matmul tolerance."""
    workloads = pkg("workloads")
    a, b = workloads.gemm_inputs()
    got = run_gemm(ctx, torch_cuda, a, b)
    exact = a.astype(np.float64) @ b.astype(np.float64)
    assert tf32.normwise_error(got, exact) <= NORMWISE
    ok, bad, err = refs.allclose_report(got, exact.astype(np.float32), 1e-3, 1e-3)
    assert ok, (bad, err)
    # size-independent checksum: column sums of C equal (1^T A) B
    colsum = (a.astype(np.float64).sum(axis=0) @ b.astype(np.float64))
    np.testing.assert_allclose(got.astype(np.float64).sum(axis=0), colsum, rtol=1e-4, atol=1e-2)


@pytest.mark.parametrize("variant", [0, 1, 2, 3])
@pytest.mark.parametrize("m,n,k", [(300, 520, 200), (128, 1024, 512), (1000, 257, 96)])
def test_gemm_every_variant(ctx, torch_cuda, variant, m, n, k):
    """Each tile/swizzle/stage variant gives the same normwise accuracy."""
    rng = np.random.default_rng(variant * 1000 + m + n + k)
    a = rng.uniform(-1, 1, (m, k)).astype(np.float32)
    b = rng.uniform(-1, 1, (k, n)).astype(np.float32)
    ctx.set_gemm_variant(variant)
    ctx.set_gemm_fused_split(0)  # variants select pre-pass kernels
    try:
        got = run_gemm(ctx, torch_cuda, a, b)
    finally:
        ctx.set_gemm_variant(1)
        ctx.set_gemm_fused_split(1)
    assert tf32.normwise_error(got, a.astype(np.float64) @ b.astype(np.float64)) <= NORMWISE


FUSED_CASES = [
    (4096, 4096, 4096, 0), (1000, 1000, 776, 1), (300, 520, 200, 0), (257, 384, 1000, 0), (130, 96, 48, 1),
    (130, 96, 48, 0), (64, 128, 16, 0), (33, 200, 20, 1), (512, 200, 36, 0), (2048, 4000, 300, 1),
    (4097, 1000, 776, 1),  # mode 1 takes the pre-pass kernel: one wave of 256-wide tiles
    # short, wide outputs (row shards of a multi-GPU GEMM): mode 1 takes the
    # transposed orientation (B split in the kernel, A pre-split)
    (512, 4096, 4096, 0), (1024, 4096, 1024, 0), (300, 2000, 1000, 1), (200, 1000, 64, 0), (130, 128, 48, 0),
]


@pytest.mark.parametrize("m,n,k,b_layout", FUSED_CASES)
def test_gemm_split_modes_match_float64_and_each_other(ctx, torch_cuda, m, n, k, b_layout):
    """The three split placements (0: pre-pass for A and B; 3: A split into
    TMEM inside the kernel, B pre-split; 2: the transposed orientation, B split
    into TMEM inside the kernel -- read MN-major from a [K, N] B or K-major
    from an [N, K] B -- A pre-split, C written transposed) and the default
    choice among them (1) against float64, the 3xTF32 model and each other on
    the same inputs.  Shapes cover ragged M, N and K, N <= 128, K = 16 and
    short wide outputs."""
    rng = np.random.default_rng(m * 31 + n * 7 + k + b_layout)
    a = rng.uniform(-1, 1, (m, k)).astype(np.float32)
    b = rng.uniform(-1, 1, (k, n) if b_layout == 0 else (n, k)).astype(np.float32)
    bias = rng.uniform(-0.5, 0.5, n).astype(np.float32)
    got = {}
    try:
        for mode in (0, 1, 2, 3):
            ctx.set_gemm_fused_split(mode)
            got[mode] = run_gemm(ctx, torch_cuda, a, b, b_layout=b_layout, bias=bias, relu=True)
    finally:
        ctx.set_gemm_fused_split(1)
    bm = b if b_layout == 0 else b.T
    rows = np.arange(m) if m <= 512 else np.random.default_rng(1).choice(m, 256, replace=False)
    exact = np.maximum(a[rows].astype(np.float64) @ bm.astype(np.float64) + bias, 0.0)
    model = np.maximum(tf32.gemm_3xtf32(a, bm) + bias, 0.0) if m * n * k <= 1 << 24 else None
    for mode in (1, 2, 3):
        assert tf32.normwise_error(got[mode][rows], exact) <= NORMWISE, mode
        # the same products and chunked folds on every path; the transposed
        # orientation swaps the MMA operand roles, which may reorder the
        # in-instruction sum of each 8-wide step (measured 1.3e-7 at 4096^3)
        assert tf32.normwise_error(got[mode], got[0]) <= 5e-7, mode
        if model is not None:
            assert tf32.normwise_error(got[mode], model) <= 2e-6, mode


def test_gemm_fused_split_special_values(ctx, torch_cuda):
    """Max-finite times zero stays 0 and infinities propagate through the
    in-kernel split as through the pre-pass split."""
    a = np.full((128, 32), np.finfo(np.float32).max, dtype=np.float32)
    b = np.zeros((32, 64), dtype=np.float32)
    np.testing.assert_array_equal(run_gemm(ctx, torch_cuda, a, b), np.zeros((128, 64), np.float32))
    # inf * (B's lo half = 0) is NaN in the hi*lo term, as in the reference's
    # 3xTF32 model; the in-kernel split must match the pre-pass split exactly.
    a = np.ones((128, 32), dtype=np.float32)
    a[5, 3] = np.inf
    a[9, 0] = np.nan
    b = np.ones((32, 64), dtype=np.float32)
    b[2, 7] = 1.5
    got = {}
    try:
        for mode in (0, 1, 2, 3):
            ctx.set_gemm_fused_split(mode)
            got[mode] = run_gemm(ctx, torch_cuda, a, b)
    finally:
        ctx.set_gemm_fused_split(1)
    for mode in (1, 2, 3):
        np.testing.assert_array_equal(got[mode], got[0])
    got = got[1]
    finite = np.setdiff1d(np.arange(128), [5, 9])
    np.testing.assert_array_equal(got[finite], (a[finite].astype(np.float64) @ b).astype(np.float32))


@pytest.mark.parametrize("m,n,k,b_layout", [(3, 33, 33, 0), (300, 520, 200, 0), (1000, 257, 96, 1),
                                            (4096, 1024, 512, 0)])
def test_gemm_scaled_divides_before_the_epilogue(ctx, torch_cuda, m, n, k, b_layout):
    """b2k_gemm_tf32x3_scaled: C = relu((A B) / div + bias), the divisor read
    from a one-element device buffer or given by value."""
    torch = torch_cuda
    rng = np.random.default_rng(m + n + k)
    a = rng.uniform(-1, 1, (m, k)).astype(np.float32)
    b = rng.uniform(-1, 1, (k, n) if b_layout == 0 else (n, k)).astype(np.float32)
    bias = rng.uniform(-0.5, 0.5, n).astype(np.float32)
    bm = (b if b_layout == 0 else b.T).astype(np.float64)
    div = np.float32(5.7445626)  # sqrt(33)
    da, db, dbias = dev(torch, a), dev(torch, b), dev(torch, bias)
    ddiv = dev(torch, np.array([div], np.float32))
    exact = np.maximum(a.astype(np.float64) @ bm / np.float64(div) + bias, 0.0)
    for by_buffer in (True, False):
        dc = torch.full((m, n), float("nan"), dtype=torch.float32, device="cuda")
        ctx.gemm_scaled(da.data_ptr(), db.data_ptr(), dc.data_ptr(), m, n, k, b_layout=b_layout,
                        div_ptr=ddiv.data_ptr() if by_buffer else 0, div_value=1.0 if by_buffer else float(div),
                        bias=dbias.data_ptr(), relu=True)
        ctx.sync()
        got = dc.cpu().numpy()
        assert tf32.normwise_error(got, exact) <= NORMWISE, by_buffer
        ok, bad, err = refs.allclose_report(got, exact.astype(np.float32), 1e-3, 1e-3)
        assert ok, (bad, err)


def test_gemm_scaled_with_unit_divisor_equals_gemm(ctx, torch_cuda):
    """Dividing by a buffer holding 1 changes no bit of the pre-pass GEMM."""
    torch = torch_cuda
    rng = np.random.default_rng(11)
    a, b = rng.uniform(-1, 1, (640, 300)).astype(np.float32), rng.uniform(-1, 1, (300, 384)).astype(np.float32)
    da, db, one = dev(torch, a), dev(torch, b), dev(torch, np.ones(1, np.float32))
    c1 = torch.empty((640, 384), device="cuda")
    c2 = torch.empty((640, 384), device="cuda")
    ctx.set_gemm_fused_split(0)
    try:
        ctx.gemm(da.data_ptr(), db.data_ptr(), c1.data_ptr(), 640, 384, 300)
        ctx.gemm_scaled(da.data_ptr(), db.data_ptr(), c2.data_ptr(), 640, 384, 300, div_ptr=one.data_ptr())
        ctx.sync()
    finally:
        ctx.set_gemm_fused_split(1)
    assert torch.equal(c1, c2)


@pytest.mark.parametrize("batch,m,n,k,b_layout", [(3, 130, 96, 48, 0), (4, 257, 300, 129, 1), (16, 128, 256, 512, 0)])
def test_gemm_batched(ctx, torch_cuda, batch, m, n, k, b_layout):
    """b2k_gemm_tf32x3_batched: each batch entry equals the single GEMM of the
    same operands bit for bit (same kernel, same split), and float64 normwise."""
    torch = torch_cuda
    runtime = pkg("runtime")
    rng = np.random.default_rng(batch * m + n + k)
    a = rng.uniform(-1, 1, (batch, m, k)).astype(np.float32)
    b = rng.uniform(-1, 1, (batch, k, n) if b_layout == 0 else (batch, n, k)).astype(np.float32)
    bias = rng.uniform(-0.5, 0.5, n).astype(np.float32)
    da, db, dbias = dev(torch, a), dev(torch, b), dev(torch, bias)
    dc = torch.full((batch, m, n), float("nan"), device="cuda")
    ctx.gemm_batched(da.data_ptr(), db.data_ptr(), dc.data_ptr(), batch, m, n, k, b_layout=b_layout,
                     bias=dbias.data_ptr(), relu=True)
    ctx.sync()
    got = dc.cpu().numpy()
    ctx.set_gemm_fused_split(0)  # the batched call runs the pre-pass kernel
    try:
        for i in range(batch):
            single = torch.empty((m, n), device="cuda")
            ctx.gemm(da[i].data_ptr(), db[i].data_ptr(), single.data_ptr(), m, n, k, b_layout=b_layout,
                     bias=dbias.data_ptr(), relu=True)
            ctx.sync()
            assert np.array_equal(got[i], single.cpu().numpy()), i
    finally:
        ctx.set_gemm_fused_split(1)
    bm = b if b_layout == 0 else np.swapaxes(b, 1, 2)
    exact = np.maximum(np.einsum("bmk,bkn->bmn", a.astype(np.float64), bm.astype(np.float64)) + bias, 0.0)
    assert tf32.normwise_error(got, exact) <= NORMWISE
    # a batch stride shorter than one matrix is refused before anything runs
    status = ctx.lib.b2k_gemm_tf32x3_batched(ctx.handle, da.data_ptr(), db.data_ptr(), dc.data_ptr(), batch, m, n, k,
                                             k, n if b_layout == 0 else k, n, m * k - 1, n * k, m * n, b_layout, None,
                                             0, None)
    with pytest.raises(runtime.B2KError):
        ctx.check(status, "b2k_gemm_tf32x3_batched")


@pytest.mark.parametrize("m,n,k,b_layout", [(257, 300, 129, 0), (130, 96, 48, 1), (1000, 1000, 776, 0)])
def test_gemm_transposed_a(ctx, torch_cuda, m, n, k, b_layout):
    """A stored [k, m] (B2K_A_KM): the same bits as the row-major A through the
    pre-pass kernel; refused by the host-array call."""
    torch = torch_cuda
    runtime = pkg("runtime")
    rng = np.random.default_rng(m + 2 * n + k)
    a = rng.uniform(-1, 1, (m, k)).astype(np.float32)
    b = rng.uniform(-1, 1, (k, n) if b_layout == 0 else (n, k)).astype(np.float32)
    bias = rng.uniform(-0.5, 0.5, n).astype(np.float32)
    da, dat, db, dbias = dev(torch, a), dev(torch, np.ascontiguousarray(a.T)), dev(torch, b), dev(torch, bias)
    bm = (b if b_layout == 0 else b.T).astype(np.float64)
    exact = np.maximum(a.astype(np.float64) @ bm + bias, 0.0)
    try:
        for mode in (0, 1, 2):
            ctx.set_gemm_fused_split(mode)
            c_t = torch.empty((m, n), device="cuda")
            ctx.gemm(dat.data_ptr(), db.data_ptr(), c_t.data_ptr(), m, n, k, b_layout=b_layout | runtime.A_KM,
                     bias=dbias.data_ptr(), relu=True)
            c = torch.empty((m, n), device="cuda")
            ctx.gemm(da.data_ptr(), db.data_ptr(), c.data_ptr(), m, n, k, b_layout=b_layout, bias=dbias.data_ptr(),
                     relu=True)
            ctx.sync()
            if mode != 1:  # same path for both storage orders: same bits
                assert torch.equal(c_t, c), mode
            assert tf32.normwise_error(c_t.cpu().numpy(), exact) <= NORMWISE, mode
    finally:
        ctx.set_gemm_fused_split(1)
    host_c = np.empty((m, n), np.float32)
    at = np.ascontiguousarray(a.T)
    with pytest.raises(runtime.B2KError):
        ctx.gemm_host(at.ctypes.data, b.ctypes.data, host_c.ctypes.data, m, n, k, b_layout=b_layout | runtime.A_KM)
