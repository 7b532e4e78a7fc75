"""Guard bands around every buffer: no kernel writes outside its output and
none writes into its inputs.

The reference's runner catches stray writes with canary images around every
buffer and input-immutability checks (tools/research_gpu.py:46-68).  The same
here, for every kernel family and the host-array calls: each operand sits
inside a larger allocation whose 256-byte margins hold a sentinel bit
pattern; after the call the margins of every buffer, and the whole of every
input, must be bit-identical to before.  Shapes have odd tails, and operands
are placed both 16-byte aligned and one float off, so the vector and the
scalar paths of each kernel run.
"""
from __future__ import annotations

import numpy as np
import pytest

from conftest import pkg

pytestmark = pytest.mark.gpu

GUARD = 64                 # floats of margin on each side (256 bytes)
SENTINEL = 0x7FBADBAD      # a NaN payload no kernel writes


class Guarded:
    """``values`` inside a device allocation with sentinel margins; ``ptr`` is
    the operand's address (``offset`` floats past a 256-byte boundary)."""

    def __init__(self, torch, values, offset=0):
        values = np.ascontiguousarray(values, dtype=np.float32)
        self.n, self.lead = values.size, GUARD + offset
        host = np.full(self.n + 2 * GUARD + offset, SENTINEL, dtype=np.uint32)
        host[self.lead:self.lead + self.n] = values.reshape(-1).view(np.uint32)
        self.before = host.copy()
        self.dev = torch.from_numpy(host.view(np.float32)).cuda()
        self.ptr = self.dev.data_ptr() + 4 * self.lead

    def after(self):
        return self.dev.cpu().numpy().view(np.uint32)

    def check_margins(self, what):
        now = self.after()
        assert np.array_equal(now[:self.lead], self.before[:self.lead]), f"{what}: write before the buffer"
        assert np.array_equal(now[self.lead + self.n:], self.before[self.lead + self.n:]), f"{what}: write past the end"

    def check_unchanged(self, what):
        assert np.array_equal(self.after(), self.before), f"{what}: input modified"

    def values(self, shape):
        return self.after()[self.lead:self.lead + self.n].view(np.float32).reshape(shape)


def run_guarded(ctx, torch, inputs, outputs, call, offset):
    """inputs / outputs: {name: array}; call(ptrs) runs the kernel."""
    g_in = {k: Guarded(torch, v, offset) for k, v in inputs.items()}
    g_out = {k: Guarded(torch, np.full(v.shape, np.nan, np.float32), offset) for k, v in outputs.items()}
    call({**{k: g.ptr for k, g in g_in.items()}, **{k: g.ptr for k, g in g_out.items()}})
    ctx.sync()
    for k, g in g_in.items():
        g.check_unchanged(k)
    for k, g in g_out.items():
        g.check_margins(k)
    return {k: g.values(outputs[k].shape) for k, g in g_out.items()}


OFFSETS = [0, 1]


@pytest.mark.parametrize("offset", OFFSETS)
def test_pointwise_and_exp(ctx, torch_cuda, offset):
    rt = pkg("runtime")
    rng = np.random.default_rng(1)
    n = 100_003
    a, b = rng.standard_normal(n).astype(np.float32), rng.standard_normal(n).astype(np.float32)
    prog = rt.make_program(2, [("add", 0, 1, 0, 0.0)], 2)
    out = run_guarded(ctx, torch_cuda, {"a": a, "b": b}, {"c": np.empty(n, np.float32)},
                      lambda p: ctx.pointwise(prog, [p["a"], p["b"]], p["c"], n), offset)
    assert np.array_equal(out["c"], a + b)
    out = run_guarded(ctx, torch_cuda, {"x": a}, {"y": np.empty(n, np.float32)},
                      lambda p: ctx.selective_exp(p["x"], p["y"], n), offset)
    assert np.isfinite(out["y"]).all()


@pytest.mark.parametrize("offset", OFFSETS)
@pytest.mark.parametrize("rows,cols", [(37, 1001), (5, 8192), (2, 70_001)])
def test_row_family(ctx, torch_cuda, offset, rows, cols):
    rt = pkg("runtime")
    x = np.random.default_rng(rows + cols).standard_normal((rows, cols)).astype(np.float32)
    w = np.random.default_rng(3).standard_normal(cols).astype(np.float32)
    y = np.empty((rows, cols), np.float32)
    r = np.empty(rows, np.float32)
    out = run_guarded(ctx, torch_cuda, {"x": x}, {"y": y}, lambda p: ctx.row_softmax(p["x"], p["y"], rows, cols),
                      offset)
    np.testing.assert_allclose(out["y"].sum(axis=1), 1.0, rtol=1e-4)
    for op in (rt.ROW_SUM, rt.ROW_MAX, rt.ROW_MIN, rt.ROW_PROD):
        run_guarded(ctx, torch_cuda, {"x": x}, {"r": r}, lambda p: ctx.row_op(op, p["x"], p["r"], rows, cols), offset)
    for op in (rt.ROW_RMSNORM, rt.ROW_L2NORM):
        run_guarded(ctx, torch_cuda, {"x": x, "w": w}, {"y": y},
                    lambda p: ctx.row_op(op, p["x"], p["y"], rows, cols, w=p["w"], ms_div=float(cols), eps=1e-6),
                    offset)


@pytest.mark.parametrize("offset", OFFSETS)
def test_axis_reduce(ctx, torch_cuda, offset):
    rt = pkg("runtime")
    x = np.random.default_rng(4).standard_normal((3, 17, 1001)).astype(np.float32)
    for op in (rt.ROW_SUM, rt.ROW_MAX):
        run_guarded(ctx, torch_cuda, {"x": x}, {"y": np.empty((3, 1001), np.float32)},
                    lambda p: ctx.axis_reduce(op, p["x"], p["y"], 3, 17, 1001), offset)


@pytest.mark.parametrize("offset", OFFSETS)
@pytest.mark.parametrize("mode", [0, 1, 2, 3])
@pytest.mark.parametrize("m,n,k,layout", [(257, 300, 129, 0), (130, 96, 48, 1), (1025, 1000, 777, 1)])
def test_gemm(ctx, torch_cuda, offset, mode, m, n, k, layout):
    rt = pkg("runtime")
    rng = np.random.default_rng(m + n + k)
    a = rng.uniform(-1, 1, (m, k)).astype(np.float32)
    b = rng.uniform(-1, 1, (k, n) if layout == 0 else (n, k)).astype(np.float32)
    bias = rng.uniform(-1, 1, n).astype(np.float32)
    div = np.array([3.0], np.float32)
    bl = rt.B_KN if layout == 0 else rt.B_NK
    ctx.set_gemm_fused_split(mode)
    try:
        out = run_guarded(ctx, torch_cuda, {"a": a, "b": b, "bias": bias}, {"c": np.empty((m, n), np.float32)},
                          lambda p: ctx.gemm(p["a"], p["b"], p["c"], m, n, k, b_layout=bl, bias=p["bias"],
                                             relu=True), offset)
        assert np.isfinite(out["c"]).all()
        run_guarded(ctx, torch_cuda, {"a": a, "b": b, "div": div}, {"c": np.empty((m, n), np.float32)},
                    lambda p: ctx.gemm_scaled(p["a"], p["b"], p["c"], m, n, k, b_layout=bl, div_ptr=p["div"]),
                    offset)
    finally:
        ctx.set_gemm_fused_split(1)


@pytest.mark.parametrize("offset", OFFSETS)
@pytest.mark.parametrize("bh,s_q,s_kv,d,dv,layout", [(2, 200, 333, 64, 40, 0), (1, 257, 129, 128, 128, 1),
                                                     (2, 65, 70, 160, 24, 0)])
def test_attention(ctx, torch_cuda, offset, bh, s_q, s_kv, d, dv, layout):
    rt = pkg("runtime")
    rng = np.random.default_rng(bh + s_q + s_kv + d)
    q = rng.standard_normal((bh, s_q, d)).astype(np.float32)
    k = rng.standard_normal((bh, s_kv, d) if layout == 0 else (bh, d, s_kv)).astype(np.float32)
    v = rng.standard_normal((bh, s_kv, dv)).astype(np.float32)
    out = run_guarded(ctx, torch_cuda, {"q": q, "k": k, "v": v}, {"o": np.empty((bh, s_q, dv), np.float32)},
                      lambda p: ctx.attention(p["q"], p["k"], p["v"], p["o"], bh, s_q, s_kv, d, dv,
                                              k_layout=rt.K_SD if layout == 0 else rt.K_DS), offset)
    assert np.isfinite(out["o"]).all()


# --------------------------------------------------------------------------- host-array calls
def host_guarded(values, offset):
    values = np.ascontiguousarray(values, dtype=np.float32)
    buf = np.full(values.size + 2 * GUARD + offset, SENTINEL, dtype=np.uint32)
    lead = GUARD + offset
    buf[lead:lead + values.size] = values.reshape(-1).view(np.uint32)
    return buf, lead


@pytest.mark.parametrize("offset", OFFSETS)
def test_host_calls(ctx, torch_cuda, offset):
    rt = pkg("runtime")
    rng = np.random.default_rng(9)
    m, n, k = 700, 333, 257
    a, b = rng.uniform(-1, 1, (m, k)).astype(np.float32), rng.uniform(-1, 1, (k, n)).astype(np.float32)
    x = rng.standard_normal((300, 1001)).astype(np.float32)
    q, kk, v = (rng.standard_normal((2, 130, 64)).astype(np.float32) for _ in range(3))
    cases = [
        ({"a": a, "b": b}, {"c": (m, n)},
         lambda p: ctx.gemm_host(p["a"], p["b"], p["c"], m, n, k)),
        ({"x": x}, {"y": x.shape},
         lambda p: ctx.row_softmax_host(p["x"], p["y"], 300, 1001)),
        ({"q": q, "k": kk, "v": v}, {"o": (2, 130, 64)},
         lambda p: ctx.attention_host(p["q"], p["k"], p["v"], p["o"], 2, 130, 130, 64, 64)),
    ]
    prog = rt.make_program(2, [("multiply", 0, 1, 0, 0.0)], 2)
    cases.append(({"a": x.reshape(-1), "b": x.reshape(-1)[::-1].copy()}, {"c": (x.size,)},
                  lambda p: ctx.pointwise_host(prog, [p["a"], p["b"]], p["c"], x.size)))
    for inputs, outputs, call in cases:
        bufs = {name: host_guarded(val, offset) for name, val in inputs.items()}
        bufs.update({name: host_guarded(np.full(shape, np.nan, np.float32), offset) for name, shape in outputs.items()})
        before = {name: buf.copy() for name, (buf, _) in bufs.items()}
        call({name: buf.ctypes.data + 4 * lead for name, (buf, lead) in bufs.items()})
        ctx.sync()
        for name, (buf, lead) in bufs.items():
            size = buf.size - 2 * GUARD - offset
            if name in inputs:
                assert np.array_equal(buf, before[name]), f"{name}: input modified"
            else:
                assert np.array_equal(buf[:lead], before[name][:lead]), f"{name}: write before the buffer"
                assert np.array_equal(buf[lead + size:], before[name][lead + size:]), f"{name}: write past the end"
                assert np.isfinite(buf[lead:lead + size].view(np.float32)).all(), name
