"""Failure detection on the GPU without a fault: a kernel whose mbarrier wait
can never complete gives up after a short cycle budget, the host reads
B2K_ETIMEOUT, and the same context then runs real work correctly."""
from __future__ import annotations

import numpy as np
import pytest

from conftest import pkg
from oracle import refs

pytestmark = pytest.mark.gpu


def test_bounded_wait_expires_with_status_and_context_survives(ctx, torch_cuda):
    runtime = pkg("runtime")
    torch = torch_cuda
    # ~1 ms at the B200's clock: the wait can only end by its budget.
    status = ctx.lib.b2k_selftest_wait_timeout(ctx.handle, 2_000_000, None)
    assert status == runtime.B2K_OK
    assert ctx.lib.b2k_stream_sync(ctx.handle, None) == runtime.B2K_ETIMEOUT
    assert b"bounded wait expired" in ctx.lib.b2k_last_error(ctx.handle)
    # the error word was cleared and the context still computes
    assert ctx.lib.b2k_stream_sync(ctx.handle, None) == runtime.B2K_OK
    rng = np.random.default_rng(5)
    a, b = rng.standard_normal(4096).astype(np.float32), rng.standard_normal(4096).astype(np.float32)
    da, db = torch.from_numpy(a).cuda(), torch.from_numpy(b).cuda()
    dc = torch.empty_like(da)
    ctx.pointwise(runtime.make_program(2, [("add", 0, 1, 0, 0.0)], 2), [da.data_ptr(), db.data_ptr()],
                  dc.data_ptr(), a.size)
    ctx.sync()
    np.testing.assert_array_equal(dc.cpu().numpy(), refs.pointwise("add", a, b))
    ga = rng.uniform(-1, 1, (256, 64)).astype(np.float32)
    gb = rng.uniform(-1, 1, (64, 256)).astype(np.float32)
    dga, dgb = torch.from_numpy(ga).cuda(), torch.from_numpy(gb).cuda()
    dgc = torch.empty((256, 256), device="cuda")
    ctx.gemm(dga.data_ptr(), dgb.data_ptr(), dgc.data_ptr(), 256, 256, 64)
    ctx.sync()
    exact = ga.astype(np.float64) @ gb.astype(np.float64)
    assert np.abs(dgc.cpu().numpy() - exact).max() / np.abs(exact).max() <= 1e-5


def test_selftest_rejects_budgets_outside_the_kernels_own(ctx):
    runtime = pkg("runtime")
    assert ctx.lib.b2k_selftest_wait_timeout(ctx.handle, 0, None) == runtime.B2K_EINVAL
    assert ctx.lib.b2k_selftest_wait_timeout(ctx.handle, 10**12, None) == runtime.B2K_EINVAL
