"""Launch overlap and host-side call plumbing on the GPU.

* programmatic dependent launch (b2k_set_pdl) changes only when kernels may
  start, never results: GEMM (both split placements) and fused attention
  are bit-identical with it on and off;
* a BoundCall re-issues exactly the call it was built from;
* b2k_timing_select restricts event timing to the selected phases.
"""
from __future__ import annotations

import numpy as np
import pytest

from conftest import pkg

pytestmark = pytest.mark.gpu


def dev(torch, a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


@pytest.mark.parametrize("mode", [1, 0])
def test_gemm_identical_with_and_without_pdl(ctx, torch_cuda, mode):
    torch = torch_cuda
    rng = np.random.default_rng(40 + mode)
    m, n, k = 1000, 700, 515
    a, b = rng.uniform(-1, 1, (m, k)).astype(np.float32), rng.uniform(-1, 1, (k, n)).astype(np.float32)
    da, db = dev(torch, a), dev(torch, b)
    out = []
    ctx.set_gemm_fused_split(mode)
    try:
        for pdl in (True, False):
            ctx.set_pdl(pdl)
            dc = torch.full((m, n), float("nan"), device="cuda")
            for _ in range(3):  # back to back: the next call's split overlaps this call's tail
                ctx.gemm(da.data_ptr(), db.data_ptr(), dc.data_ptr(), m, n, k)
            ctx.sync()
            out.append(dc.cpu().numpy())
    finally:
        ctx.set_pdl(True)
        ctx.set_gemm_fused_split(1)
    assert np.array_equal(out[0], out[1])
    assert np.isfinite(out[0]).all()


def test_attention_identical_with_and_without_pdl(ctx, torch_cuda):
    torch = torch_cuda
    rng = np.random.default_rng(44)
    bh, s, d = 4, 384, 128
    q, k, v = (rng.standard_normal((bh, s, d)).astype(np.float32) for _ in range(3))
    dq, dk, dv = dev(torch, q), dev(torch, k), dev(torch, v)
    out = []
    for pdl in (True, False):
        ctx.set_pdl(pdl)
        do = torch.full_like(dq, float("nan"))
        for _ in range(2):
            ctx.attention(dq.data_ptr(), dk.data_ptr(), dv.data_ptr(), do.data_ptr(), bh, s, s, d, d)
        ctx.sync()
        out.append(do.cpu().numpy())
    ctx.set_pdl(True)
    assert np.array_equal(out[0], out[1])


def test_bound_call_reissues_the_same_gemm(ctx, torch_cuda):
    torch = torch_cuda
    rt = pkg("runtime")
    rng = np.random.default_rng(45)
    m, n, k = 300, 200, 777
    a = rng.uniform(-1, 1, (m, k)).astype(np.float32)
    bt = rng.uniform(-1, 1, (n, k)).astype(np.float32)
    bias = rng.uniform(-1, 1, n).astype(np.float32)
    da, db, dbias = dev(torch, a), dev(torch, bt), dev(torch, bias)
    c1 = torch.empty((m, n), device="cuda")
    c2 = torch.empty((m, n), device="cuda")
    before = ctx.kernel_launches()
    ctx.gemm(da.data_ptr(), db.data_ptr(), c1.data_ptr(), m, n, k, b_layout=rt.B_NK, bias=dbias.data_ptr(),
             relu=True)
    per_call = ctx.kernel_launches() - before  # operand split, tensor-core kernel(s), fold when K is chunk-split
    assert per_call in (2, 3)
    call = ctx.gemm_call(da.data_ptr(), db.data_ptr(), c2.data_ptr(), m, n, k, b_layout=rt.B_NK,
                         bias=dbias.data_ptr(), relu=True)
    before = ctx.kernel_launches()
    call()
    call()
    assert ctx.kernel_launches() - before == 2 * per_call
    ctx.sync()
    assert torch.equal(c1, c2)


def test_bound_call_raises_on_failure(ctx):
    rt = pkg("runtime")
    call = ctx.gemm_call(0, 0, 0, 16, 16, 16)  # null buffers
    with pytest.raises(rt.B2KError):
        call()


def test_timing_select_times_only_selected_phases(ctx, torch_cuda):
    torch = torch_cuda
    m = n = k = 256
    da, db = torch.rand((m, k), device="cuda"), torch.rand((k, n), device="cuda")
    dc = torch.empty((m, n), device="cuda")
    ctx.timing_reset()
    ctx.timing(True, phases=["mma"])
    for _ in range(3):
        ctx.gemm(da.data_ptr(), db.data_ptr(), dc.data_ptr(), m, n, k)
    ctx.timing(False)
    ms, launches = ctx.timing_read("mma")
    split_ms, split_launches = ctx.timing_read("split")
    ctx.timing_reset()
    assert launches == 3 and ms > 0.0
    assert split_launches == 0 and split_ms == 0.0
