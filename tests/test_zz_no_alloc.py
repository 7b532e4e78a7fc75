"""The allocation-free GEMM entry point, b2k_gemm_tf32x3_noalloc.

Some callers cannot call cudaMalloc (embedders whose device memory belongs to
another allocator or a pre-sized pool, runtimes that plan every buffer up
front, host callbacks); for them the library offers a GEMM that
keeps its operand split in a fixed array inside the library image instead of
a context's growable scratch.  These tests call it through the C ABI twice in
a row, with different shapes, layouts and data, and check each result
against the allocating entry point, b2k_gemm_tf32x3, at the matmul
tolerance the other GEMM tests use (rtol = atol = 1e-3, and the 1e-5
normwise bound against float64).  This file sorts last so that a run which
stops at the first failure has already run every other test.
"""
from __future__ import annotations

import ctypes

import numpy as np
import pytest

from conftest import pkg
from oracle import refs, tf32

pytestmark = pytest.mark.gpu


def call_noalloc(lib, a, b, c, m, n, k, lda, ldb, ldc, layout, bias, relu):
    return lib.b2k_gemm_tf32x3_noalloc(a, b, c, m, n, k, lda, ldb, ldc, layout, bias, relu, None)


CASES = [
    # (m, n, k, b_layout, bias, relu)
    (384, 512, 320, 0, False, False),
    (300, 200, 77, 1, True, True),
]


def test_noalloc_matches_allocating_gemm_on_consecutive_calls(ctx, torch_cuda):
    torch = torch_cuda
    runtime = pkg("runtime")
    lib = runtime.library()
    for call, (m, n, k, layout, with_bias, relu) in enumerate(CASES):
        rng = np.random.default_rng(100 + call)
        a = rng.standard_normal((m, k)).astype(np.float32)
        b = rng.standard_normal((k, n) if layout == 0 else (n, k)).astype(np.float32)
        bias = rng.uniform(-0.5, 0.5, n).astype(np.float32) if with_bias else None
        da, db = torch.from_numpy(a).cuda(), torch.from_numpy(b).cuda()
        dbias = torch.from_numpy(bias).cuda() if with_bias else None
        bias_ptr = dbias.data_ptr() if with_bias else 0
        ldb = n if layout == 0 else k
        # existing entry point (context scratch)
        c_ref = torch.full((m, n), float("nan"), device="cuda")
        ctx.gemm(da.data_ptr(), db.data_ptr(), c_ref.data_ptr(), m, n, k, b_layout=layout,
                 bias=bias_ptr, relu=relu)
        # allocation-free entry point (fixed scratch array)
        c_new = torch.full((m, n), float("nan"), device="cuda")
        status = call_noalloc(lib, da.data_ptr(), db.data_ptr(), c_new.data_ptr(), m, n, k, k, ldb, n,
                              layout, bias_ptr or None, int(relu))
        assert status == runtime.B2K_OK, status
        torch.cuda.synchronize()
        got, want = c_new.cpu().numpy(), c_ref.cpu().numpy()
        ok, bad, err = refs.allclose_report(got, want, 1e-3, 1e-3)
        assert ok, (call, bad, err)
        bt = b.T if layout == 0 else b
        exact = a.astype(np.float64) @ bt.astype(np.float64).T
        if with_bias:
            exact = exact + bias
        if relu:
            exact = np.maximum(exact, 0.0)
        assert tf32.normwise_error(got, exact) <= 1e-5, call


def test_noalloc_rejects_problems_beyond_its_scratch(ctx, torch_cuda):
    runtime = pkg("runtime")
    lib = runtime.library()
    # 2 * (4096 + 4096) * 4096 * 4 bytes = 256 MiB of split operands > 32 MiB
    m = n = k = 4096
    assert 2 * (m + n) * k * 4 > runtime.NOALLOC_SCRATCH_BYTES
    dummy = torch_cuda.empty(16, device="cuda")
    p = dummy.data_ptr()
    status = call_noalloc(lib, p, p, p, m, n, k, k, n, n, 0, None, 0)
    assert status == runtime.B2K_ESCRATCH
    # A K so large that 2 * (m + n) * round_up(k, 32) would wrap int64 to a
    # small number: refused before any size arithmetic, nothing launched.
    status = call_noalloc(lib, p, p, p, 1, 1, 1 << 62, 1 << 62, 1, 1, 0, None, 0)
    assert status == runtime.B2K_EINVAL
    torch_cuda.cuda.synchronize()


def test_noalloc_status_reads_and_clears_the_device_word(ctx, torch_cuda):
    """b2k_gemm_noalloc_status: after completed calls with no expired wait it
    returns B2K_OK (and again on a second query); device indices outside the
    machine return B2K_EINVAL; the calling thread's current device is kept."""
    torch = torch_cuda
    runtime = pkg("runtime")
    lib = runtime.library()
    m, n, k = 256, 384, 96
    rng = np.random.default_rng(7)
    da = torch.from_numpy(rng.standard_normal((m, k)).astype(np.float32)).cuda()
    db = torch.from_numpy(rng.standard_normal((k, n)).astype(np.float32)).cuda()
    dc = torch.empty((m, n), device="cuda")
    assert call_noalloc(lib, da.data_ptr(), db.data_ptr(), dc.data_ptr(), m, n, k, k, n, n, 0, None, 0) == 0
    torch.cuda.synchronize()
    device = torch.cuda.current_device()
    assert lib.b2k_gemm_noalloc_status(device) == runtime.B2K_OK
    assert lib.b2k_gemm_noalloc_status(device) == runtime.B2K_OK
    assert torch.cuda.current_device() == device
    assert lib.b2k_gemm_noalloc_status(-1) == runtime.B2K_EINVAL
    assert lib.b2k_gemm_noalloc_status(torch.cuda.device_count()) == runtime.B2K_EINVAL
