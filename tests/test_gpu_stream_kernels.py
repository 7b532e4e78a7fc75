"""GPU parity of the bandwidth-bound kernels (pointwise programs, row softmax,
selective exp) through the C ABI, against the float64 oracle."""
from __future__ import annotations

import numpy as np
import pytest

from conftest import pkg
from oracle import refs, sexp

pytestmark = pytest.mark.gpu


def dev(torch, array):
    return torch.from_numpy(np.ascontiguousarray(array)).cuda()


def run_program(ctx, torch, program, arrays, n):
    inputs = [dev(torch, a) for a in arrays]
    out = torch.empty(n, dtype=torch.float32, device="cuda")
    ctx.pointwise(program, [t.data_ptr() for t in inputs], out.data_ptr(), n)
    ctx.sync()
    return out.cpu().numpy()


@pytest.mark.parametrize("n", [1, 3, 4, 127, 128, 1024, 4099, 65537, 1 << 20])
def test_add_bit_exact(ctx, torch_cuda, n):
    runtime = pkg("runtime")
    rng = np.random.default_rng(n)
    a, b = rng.standard_normal(n).astype(np.float32), rng.standard_normal(n).astype(np.float32)
    prog = runtime.make_program(2, [("add", 0, 1, 0, 0.0)], 2)
    got = run_program(ctx, torch_cuda, prog, [a, b], n)
    np.testing.assert_array_equal(got, refs.pointwise("add", a, b))


def test_add_baseline_size_bit_exact(ctx, torch_cuda):
    runtime, workloads = pkg("runtime"), pkg("workloads")
    a, b = workloads.add_inputs()
    prog = runtime.make_program(2, [("add", 0, 1, 0, 0.0)], 2)
    got = run_program(ctx, torch_cuda, prog, [a, b], a.size)
    np.testing.assert_array_equal(got, (a + b).astype(np.float32))


def test_add_unaligned_views(ctx, torch_cuda):
    """Offsets that break 16-byte alignment take the scalar path and stay exact."""
    runtime = pkg("runtime")
    torch = torch_cuda
    n = 1001
    a = torch.randn(n + 3, device="cuda")
    b = torch.randn(n + 3, device="cuda")
    out = torch.empty(n + 3, device="cuda")
    prog = runtime.make_program(2, [("add", 0, 1, 0, 0.0)], 2)
    ctx.pointwise(prog, [a[1:].data_ptr(), b[2:].data_ptr()], out[3:].data_ptr(), n)
    ctx.sync()
    expect = (a[1:1 + n].cpu().numpy() + b[2:2 + n].cpu().numpy()).astype(np.float32)
    np.testing.assert_array_equal(out[3:3 + n].cpu().numpy(), expect)


def test_programs_scale_shift_and_relu_mul(ctx, torch_cuda):
    runtime = pkg("runtime")
    rng = np.random.default_rng(7)
    n = 4096
    x, y = rng.standard_normal(n).astype(np.float32), rng.standard_normal(n).astype(np.float32)
    # p02 shape: add(add_c1, multiply(mul_c1, x)) with two broadcast scalars
    prog = runtime.make_program(3, [("multiply", 0, 2, 0, 0.0), ("add", 1, 3, 0, 0.0)], 4, broadcast=(0, 1))
    got = run_program(ctx, torch_cuda, prog, [np.array([2.0], np.float32), np.array([1.0], np.float32), x], n)
    ok, bad, err = refs.allclose_report(got, refs.pointwise("scale_shift", x, np.array([2.0]), np.array([1.0])),
                                        1e-6, 1e-6)
    assert ok, (bad, err)
    # p03 shape: multiply(y, relu(x)), rtol = atol = 0
    prog = runtime.make_program(2, [("relu", 0, 0, 0, 0.0), ("multiply", 1, 2, 0, 0.0)], 3)
    got = run_program(ctx, torch_cuda, prog, [x, y], n)
    np.testing.assert_array_equal(got, refs.pointwise("relu_mul", x, y))


@pytest.mark.parametrize("rows,cols", [(64, 256), (5, 257), (3, 127), (32, 31), (16, 8192), (2, 20000), (7, 4096)])
def test_row_softmax_matches_float64(ctx, torch_cuda, rows, cols):
    rng = np.random.default_rng(rows * 100003 + cols)
    x = (rng.standard_normal((rows, cols)) * 4).astype(np.float32)
    xd = dev(torch_cuda, x)
    y = torch_cuda.empty_like(xd)
    ctx.row_softmax(xd.data_ptr(), y.data_ptr(), rows, cols)
    ctx.sync()
    ok, bad, err = refs.allclose_report(y.cpu().numpy(), refs.softmax(x), 1e-3, 1e-5)
    assert ok, (bad, err)


def test_row_softmax_baseline_config(ctx, torch_cuda):
    """4096 x 8192, N(0, 16) with 1 % of entries at -100 (checked on every row)."""
    workloads = pkg("workloads")
    x = workloads.softmax_input()
    xd = dev(torch_cuda, x)
    y = torch_cuda.empty_like(xd)
    ctx.row_softmax(xd.data_ptr(), y.data_ptr(), *x.shape)
    ctx.sync()
    got = y.cpu().numpy()
    ok, bad, err = refs.allclose_report(got, refs.softmax(x), 1e-3, 1e-5)
    assert ok, (bad, err)
    # size-independent property: every row sums to one
    np.testing.assert_allclose(got.astype(np.float64).sum(axis=1), 1.0, rtol=1e-5)


def test_selective_exp_subnormal_range(ctx, torch_cuda):
    """exp over [-104, -86] keeps subnormal results within the method's bound."""
    x = np.linspace(-110.0, 5.0, 1 << 16, dtype=np.float32)
    xd = dev(torch_cuda, x)
    y = torch_cuda.empty_like(xd)
    ctx.selective_exp(xd.data_ptr(), y.data_ptr(), x.size)
    ctx.sync()
    got = y.cpu().numpy()
    report = sexp.check_against_exp(x, got)
    assert report["ok"], report
    sub = (x > -103.0) & (x < -88.0)
    assert np.all(got[sub] > 0.0), "subnormal results were flushed"


@pytest.mark.parametrize("rows,cols", [(4096, 8192), (64, 1024), (7, 3), (3, 20000)])
def test_row_norms_match_float64(ctx, torch_cuda, rows, cols):
    runtime = pkg("runtime")
    rng = np.random.default_rng(rows + cols)
    x = rng.standard_normal((rows, cols)).astype(np.float32)
    w = rng.standard_normal(cols).astype(np.float32)
    dx, dw = dev(torch_cuda, x), dev(torch_cuda, w)
    y = torch_cuda.empty_like(dx)
    ctx.row_op(runtime.ROW_RMSNORM, dx.data_ptr(), y.data_ptr(), rows, cols, ms_div=float(cols), eps=1e-5,
               w=dw.data_ptr())
    ctx.sync()
    ok, bad, err = refs.allclose_report(y.cpu().numpy(), refs.rmsnorm(x, w, 1e-5), 1e-3, 1e-4)
    assert ok, (bad, err)
    ctx.row_op(runtime.ROW_L2NORM, dx.data_ptr(), y.data_ptr(), rows, cols)
    ctx.sync()
    ok, bad, err = refs.allclose_report(y.cpu().numpy(), refs.l2norm(x), 1e-3, 1e-4)
    assert ok, (bad, err)


@pytest.mark.parametrize("n", [1, 1000, 65536, 65537, 1 << 24])
def test_whole_array_sum_deterministic(ctx, torch_cuda, n):
    runtime = pkg("runtime")
    x = np.random.default_rng(n).standard_normal(n).astype(np.float32)
    dx = dev(torch_cuda, x)
    y = torch_cuda.empty(1, device="cuda")
    results = []
    for _ in range(2):
        ctx.row_op(runtime.ROW_SUM, dx.data_ptr(), y.data_ptr(), 1, n)
        ctx.sync()
        results.append(y.cpu().numpy().copy())
    assert results[0].tobytes() == results[1].tobytes()  # fixed combination order
    ok, bad, err = refs.allclose_report(results[0], refs.array_sum(x), 1e-4, 1e-3)
    assert ok, (bad, err)


def test_row_sums_and_means(ctx, torch_cuda):
    runtime = pkg("runtime")
    x = np.random.default_rng(4).standard_normal((64, 512)).astype(np.float32)
    dx = dev(torch_cuda, x)
    y = torch_cuda.empty(64, device="cuda")
    ctx.row_op(runtime.ROW_SUM, dx.data_ptr(), y.data_ptr(), 64, 512, sum_div=512.0)
    ctx.sync()
    ok, bad, err = refs.allclose_report(y.cpu().numpy(), (refs.row_sum(x) / 512).astype(np.float32), 1e-4, 1e-6)
    assert ok, (bad, err)


@pytest.mark.parametrize("rows,cols", [(1, 127), (3, 4), (64, 1000), (5, 70000)])
def test_row_max_min_prod(ctx, torch_cuda, rows, cols):
    """Non-additive row folds: max and min exact, product within FP32
    rounding of a fixed-order tree (inputs near 1 keep it finite)."""
    runtime = pkg("runtime")
    rng = np.random.default_rng(rows * 7 + cols)
    x = rng.standard_normal((rows, cols)).astype(np.float32)
    x[:, ::7] = -np.inf if cols > 8 else x[:, ::7]  # max must skip -inf entries
    near_one = (1.0 + rng.uniform(-1e-3, 1e-3, (rows, cols))).astype(np.float32)
    dx, dn = dev(torch_cuda, x), dev(torch_cuda, near_one)
    y = torch_cuda.empty(rows, device="cuda")
    ctx.row_op(runtime.ROW_MAX, dx.data_ptr(), y.data_ptr(), rows, cols)
    ctx.sync()
    assert np.array_equal(y.cpu().numpy(), x.max(axis=1))
    ctx.row_op(runtime.ROW_MIN, dx.data_ptr(), y.data_ptr(), rows, cols)
    ctx.sync()
    assert np.array_equal(y.cpu().numpy(), x.min(axis=1))
    ctx.row_op(runtime.ROW_PROD, dn.data_ptr(), y.data_ptr(), rows, cols)
    ctx.sync()
    want = near_one.astype(np.float64).prod(axis=1)
    np.testing.assert_allclose(y.cpu().numpy(), want, rtol=cols * 2.0 ** -23, atol=0)
    # the same launch twice gives the same bits (fixed combine order)
    first = y.clone()
    ctx.row_op(runtime.ROW_PROD, dn.data_ptr(), y.data_ptr(), rows, cols)
    ctx.sync()
    assert torch_cuda.equal(first, y)


@pytest.mark.parametrize("batch,s,cols", [(2, 9, 64), (3, 1, 64), (1, 2, 32), (5, 300, 1000), (70000, 3, 5),
                                          (4, 0, 7)])
def test_axis_reduce(ctx, torch_cuda, batch, s, cols):
    """Folds over the middle axis of [batch, s, cols]: the sum (and a mean
    through a divisor buffer) in order over s, max / min exact, the product
    within FP32 rounding; s = 0 gives each fold's identity."""
    runtime = pkg("runtime")
    rng = np.random.default_rng(batch + 7 * s + cols)
    x = rng.standard_normal((batch, s, cols)).astype(np.float32)
    near_one = (1.0 + rng.uniform(-1e-3, 1e-3, (batch, s, cols))).astype(np.float32)
    dx, dn = dev(torch_cuda, x), dev(torch_cuda, near_one)
    y = torch_cuda.full((batch, cols), float("nan"), device="cuda")

    def run(op, src, **kw):
        ctx.axis_reduce(op, src.data_ptr(), y.data_ptr(), batch, s, cols, **kw)
        ctx.sync()
        return y.cpu().numpy()

    seq = np.zeros((batch, cols), np.float32)  # the serial FP32 fold the IR describes
    for i in range(s):
        seq = seq + x[:, i, :]
    assert np.array_equal(run(runtime.ROW_SUM, dx), seq)
    div = dev(torch_cuda, np.array([max(s, 1)], np.float32))
    assert np.array_equal(run(runtime.ROW_SUM, dx, div_ptr=div.data_ptr()), seq / np.float32(max(s, 1)))
    assert np.array_equal(run(runtime.ROW_SUM, dx, div=4.0), seq / np.float32(4.0))
    want_max = x.max(axis=1) if s else np.full((batch, cols), -np.inf, np.float32)
    want_min = x.min(axis=1) if s else np.full((batch, cols), np.inf, np.float32)
    assert np.array_equal(run(runtime.ROW_MAX, dx), want_max)
    assert np.array_equal(run(runtime.ROW_MIN, dx), want_min)
    np.testing.assert_allclose(run(runtime.ROW_PROD, dn), near_one.astype(np.float64).prod(axis=1),
                               rtol=max(s, 1) * 2.0 ** -23, atol=0)


def test_axis_reduce_rejects_bad_arguments(ctx, torch_cuda):
    runtime = pkg("runtime")
    y = torch_cuda.empty(4, device="cuda")
    with pytest.raises(runtime.B2KError):
        ctx.axis_reduce(runtime.ROW_RMSNORM, y.data_ptr(), y.data_ptr(), 1, 1, 4)
    with pytest.raises(runtime.B2KError):
        ctx.axis_reduce(runtime.ROW_SUM, y.data_ptr(), y.data_ptr(), 1, -1, 4)


@pytest.mark.parametrize("n", [260, 1 << 20, 1000003])
def test_pointwise_windows(ctx, torch_cuda, n):
    """Input streams read at element offsets (shifted windows): out[i] =
    x[i + 1] * y[i + 2] + x[i], bit-exact against NumPy, through the device
    entry point and the host-array call."""
    runtime = pkg("runtime")
    rng = np.random.default_rng(n)
    x = rng.standard_normal(n + 1).astype(np.float32)
    y = rng.standard_normal(n + 2).astype(np.float32)
    prog = runtime.make_program(3, [("multiply", 0, 1, 0, 0.0), ("add", 3, 2, 0, 0.0)], 4, offsets=(1, 2, 0))
    want = x[1:n + 1] * y[2:n + 2] + x[:n]
    dx, dy = dev(torch_cuda, x), dev(torch_cuda, y)
    out = torch_cuda.empty(n, device="cuda")
    ctx.pointwise(prog, [dx.data_ptr(), dy.data_ptr(), dx.data_ptr()], out.data_ptr(), n)
    ctx.sync()
    assert np.array_equal(out.cpu().numpy(), want)
    got = np.empty(n, np.float32)
    ctx.pointwise_host(prog, [x.ctypes.data, y.ctypes.data, x.ctypes.data], got.ctypes.data, n)
    ctx.sync()
    assert np.array_equal(got, want)
    bad = runtime.make_program(1, [("copy", 0, 0, 0, 0.0)], 1, offsets=(-1,))
    with pytest.raises(runtime.B2KError):
        ctx.pointwise(bad, [dx.data_ptr()], out.data_ptr(), n)
