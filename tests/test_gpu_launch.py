"""b2k_launch: the runner's positional-argument launch (cuLaunchKernel params
convention, tools/local_runner.py:296-324) with a kernel descriptor.  Each
kind against its direct entry point, argument slots mixing buffers and f32
scalars, and validation failures that launch nothing."""
from __future__ import annotations

import numpy as np
import pytest

from conftest import pkg
from oracle import refs, tf32

pytestmark = pytest.mark.gpu


def dev(torch, a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def test_gemm_by_descriptor_with_scalar_slots(ctx, torch_cuda):
    rt = pkg("runtime")
    rng = np.random.default_rng(21)
    m, n, k = 300, 200, 96
    a = rng.uniform(-1, 1, (m, k)).astype(np.float32)
    bt = rng.uniform(-1, 1, (n, k)).astype(np.float32)
    bias = rng.uniform(-0.5, 0.5, n).astype(np.float32)
    da, db, dbias = dev(torch_cuda, a), dev(torch_cuda, bt), dev(torch_cuda, bias)
    dc = torch_cuda.full((m, n), float("nan"), device="cuda")
    # positional order as a meta.json might list it: a scalar, C, bias, B, another scalar, A
    args = [3.5, dc.data_ptr(), dbias.data_ptr(), db.data_ptr(), -1.0, da.data_ptr()]
    desc = rt.make_desc(rt.KIND_GEMM, {0: 5, 1: 3, 2: 1, 3: 2}, dims=(m, n, k, k, k, n), flags=(rt.B_NK, 1))
    ctx.launch(desc, args)
    ctx.sync()
    exact = np.maximum(a.astype(np.float64) @ bt.astype(np.float64).T + bias, 0.0)
    assert tf32.normwise_error(dc.cpu().numpy(), exact) <= 1e-5


def test_row_ops_softmax_pointwise_attention_by_descriptor(ctx, torch_cuda):
    rt = pkg("runtime")
    torch = torch_cuda
    rng = np.random.default_rng(22)
    x = rng.standard_normal((64, 256)).astype(np.float32)
    w = rng.standard_normal(256).astype(np.float32)
    dx, dw, dy = dev(torch, x), dev(torch, w), torch.empty((64, 256), device="cuda")
    eps = dev(torch, np.array([1e-5], np.float32))
    ctx.launch(rt.make_desc(rt.KIND_ROW_OP, {0: 2, 1: 0, 2: 1, 5: 3}, dims=(64, 256, 256, 256),
                            flags=(rt.ROW_RMSNORM,), values=(1.0, 256.0, 0.0)),
               [dy.data_ptr(), dw.data_ptr(), dx.data_ptr(), eps.data_ptr()])
    ctx.sync()
    ok, bad, err = refs.allclose_report(dy.cpu().numpy(), refs.rmsnorm(x, w, 1e-5), 1e-3, 1e-4)
    assert ok, (bad, err)
    ctx.launch(rt.make_desc(rt.KIND_ROW_SOFTMAX, {0: 1, 1: 0}, dims=(64, 256, 256, 256)), [dy.data_ptr(), dx.data_ptr()])
    ctx.sync()
    ok, bad, err = refs.allclose_report(dy.cpu().numpy(), refs.softmax(x), 1e-3, 1e-5)
    assert ok, (bad, err)
    a, b = rng.standard_normal(1001).astype(np.float32), rng.standard_normal(1001).astype(np.float32)
    da, db, dc = dev(torch, a), dev(torch, b), torch.empty(1001, device="cuda")
    prog = rt.make_program(2, [("add", 0, 1, 0, 0.0)], 2)
    ctx.launch(rt.make_desc(rt.KIND_POINTWISE, {0: 2, 1: 0, rt.ROLE_PW_OUT: 1}, dims=(1001,), program=prog),
               [db.data_ptr(), dc.data_ptr(), da.data_ptr()])
    ctx.sync()
    np.testing.assert_array_equal(dc.cpu().numpy(), refs.pointwise("add", b, a))
    q, kt, v = (rng.standard_normal(s).astype(np.float32) for s in ((128, 64), (64, 128), (128, 64)))
    dq, dkt, dv, do = dev(torch, q), dev(torch, kt), dev(torch, v), torch.empty((128, 64), device="cuda")
    div = dev(torch, np.array([8.0], np.float32))
    ctx.launch(rt.make_desc(rt.KIND_ATTENTION, {0: 0, 1: 1, 2: 2, 3: 4, 4: 3}, dims=(1, 128, 128, 64, 64),
                            flags=(rt.K_DS,)),
               [dq.data_ptr(), dkt.data_ptr(), dv.data_ptr(), div.data_ptr(), do.data_ptr()])
    ctx.sync()
    ok, bad, err = refs.allclose_report(do.cpu().numpy(), refs.attention(q, kt, v, 8.0), 1e-3, 1e-4)
    assert ok, (bad, err)


def test_bad_descriptors_fail_before_launching(ctx, torch_cuda):
    rt = pkg("runtime")
    buf = torch_cuda.zeros(1024, device="cuda")
    before = ctx.kernel_launches()
    cases = [
        rt.make_desc(rt.KIND_GEMM, {0: 0, 1: 1, 2: 7}, dims=(8, 8, 8, 8, 8, 8)),      # role past nargs
        rt.make_desc(rt.KIND_GEMM, {0: 0, 1: 1}, dims=(8, 8, 8, 8, 8, 8)),            # C missing
        rt.make_desc(99, {0: 0}),                                                      # unknown kind
        rt.make_desc(rt.KIND_POINTWISE, {0: 0, rt.ROLE_PW_OUT: 1}, dims=(8,)),        # no program
        rt.make_desc(rt.KIND_ROW_SOFTMAX, {0: 0, 1: 1}, dims=(4, 16, 16, 16)),       # null buffer slot
    ]
    arg_sets = [[buf.data_ptr()] * 3, [buf.data_ptr()] * 3, [buf.data_ptr()], [buf.data_ptr()] * 2,
                [buf.data_ptr(), 0]]
    for desc, args in zip(cases, arg_sets):
        with pytest.raises(rt.B2KError) as info:
            ctx.launch(desc, args)
        assert info.value.status == rt.B2K_EINVAL
    assert ctx.lib.b2k_launch(ctx.handle, None, None, 0, None) == rt.B2K_EINVAL
    assert ctx.kernel_launches() == before
