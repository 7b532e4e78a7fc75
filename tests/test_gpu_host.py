"""GPU parity of the pipelined host-array calls (b2k_*_host).

Each host call must equal the device entry point of the same name bit for
bit: the slabs run the same kernels on the same values, only the copies are
overlapped.  Sizes are chosen so that several cases cut into more than one
slab (slabs hold 4 to 16 MB of input), and pitched host rows, a broadcast
pointwise input, both B layouts, bias + ReLU and the three GEMM split modes
are covered.  The reference for the device paths themselves is the float64
oracle in the other test files.
"""
from __future__ import annotations

import numpy as np
import pytest

from conftest import pkg

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def session(torch_cuda):
    s = pkg("api").Session(0)
    yield s
    s.close()


def pinned_copy(session, x):
    p = session.pinned(x.shape)
    p[...] = x
    return p


@pytest.mark.parametrize("rows,cols", [(1000, 3000), (2048, 2048), (3, 5)])
def test_row_softmax_host_equals_device(session, torch_cuda, rows, cols):
    torch = torch_cuda
    x = np.random.default_rng(rows + cols).normal(0, 4, (rows, cols)).astype(np.float32)
    hx = pinned_copy(session, x)
    hy = session.pinned(x.shape)
    session.row_softmax_host(hx, hy)
    session.sync()
    dx = torch.from_numpy(x).cuda()
    dy = torch.empty_like(dx)
    session.ctx.row_softmax(dx.data_ptr(), dy.data_ptr(), rows, cols)
    session.ctx.sync()
    assert np.array_equal(hy, dy.cpu().numpy())


def test_row_softmax_host_pitched_rows(session, torch_cuda):
    torch = torch_cuda
    rows, cols, ld = 700, 1000, 1003
    x = np.random.default_rng(5).normal(0, 3, (rows, ld)).astype(np.float32)
    y = np.full((rows, ld + 2), np.nan, np.float32)
    session.ctx.row_softmax_host(x.ctypes.data, y.ctypes.data, rows, cols, ld, ld + 2)
    session.sync()
    dx = torch.from_numpy(np.ascontiguousarray(x[:, :cols])).cuda()
    dy = torch.empty_like(dx)
    session.ctx.row_softmax(dx.data_ptr(), dy.data_ptr(), rows, cols)
    session.ctx.sync()
    assert np.array_equal(y[:, :cols], dy.cpu().numpy())
    assert np.isnan(y[:, cols:]).all()  # bytes past each row untouched


@pytest.mark.parametrize("n", [(1 << 22) + 3, 1000, 1])
def test_pointwise_host_equals_device(session, torch_cuda, n):
    torch = torch_cuda
    rt = pkg("runtime")
    rng = np.random.default_rng(n)
    a = rng.uniform(-1, 1, n).astype(np.float32)
    b = rng.uniform(-1, 1, n).astype(np.float32)
    s = np.array([1.5], np.float32)
    # (a + b) * s with s a broadcast scalar input
    prog = rt.make_program(3, [("add", 0, 1, 0, 0.0), ("multiply", 3, 2, 0, 0.0)], 4, broadcast=(2,))
    out = session.pinned((n,))
    session.pointwise_host(prog, [pinned_copy(session, a), pinned_copy(session, b), s], out)
    session.sync()
    da, db, ds = (torch.from_numpy(t).cuda() for t in (a, b, s))
    dout = torch.empty_like(da)
    session.ctx.pointwise(prog, [da.data_ptr(), db.data_ptr(), ds.data_ptr()], dout.data_ptr(), n)
    session.ctx.sync()
    assert np.array_equal(out, dout.cpu().numpy())


GEMM_CASES = [
    # m, n, k, b_layout, bias+relu, split mode
    (2304, 1024, 1024, "kn", False, 1),   # several slabs, A split into TMEM
    (1000, 520, 300, "nk", True, 1),
    (2300, 700, 777, "nk", True, 1),      # lda 777: pre-pass split of each slab
    (640, 384, 256, "kn", False, 0),
    (640, 384, 256, "kn", True, 2),       # transposed orientation: each slab splits its rows of A
    (700, 4096, 512, "kn", True, 1),      # short and wide: the default takes the transposed orientation
    (300, 1000, 640, "nk", False, 2),
    (5, 7, 3, "kn", False, 1),
    (2304, 1024, 1024, "kn", False, 3),   # A split into TMEM, forced
    (4097, 1000, 776, "nk", True, 1),     # aligned A, but the pre-pass kernel tiles in fewer waves
]


@pytest.mark.parametrize("m,n,k,layout,epi,mode", GEMM_CASES)
def test_gemm_host_equals_device(session, torch_cuda, m, n, k, layout, epi, mode):
    torch = torch_cuda
    rt = pkg("runtime")
    rng = np.random.default_rng(m + n + k)
    a = rng.uniform(-1, 1, (m, k)).astype(np.float32)
    b = rng.uniform(-1, 1, (k, n) if layout == "kn" else (n, k)).astype(np.float32)
    bias = rng.uniform(-1, 1, n).astype(np.float32) if epi else None
    session.ctx.set_gemm_fused_split(mode)
    try:
        c = session.pinned((m, n))
        session.gemm_host(pinned_copy(session, a), pinned_copy(session, b), c, b_layout=layout,
                          bias=pinned_copy(session, bias) if epi else None, relu=epi)
        session.sync()
        da, db = torch.from_numpy(a).cuda(), torch.from_numpy(b).cuda()
        dbias = torch.from_numpy(bias).cuda() if epi else None
        dc = torch.empty((m, n), dtype=torch.float32, device="cuda")
        session.ctx.gemm(da.data_ptr(), db.data_ptr(), dc.data_ptr(), m, n, k,
                         b_layout=rt.B_KN if layout == "kn" else rt.B_NK,
                         bias=dbias.data_ptr() if epi else 0, relu=epi)
        session.ctx.sync()
    finally:
        session.ctx.set_gemm_fused_split(1)
    assert np.array_equal(c, dc.cpu().numpy())


@pytest.mark.parametrize("bh,s,d,layout", [(40, 512, 128, "sd"), (3, 300, 64, "ds"), (1, 1, 32, "sd")])
def test_attention_host_equals_device(session, torch_cuda, bh, s, d, layout):
    torch = torch_cuda
    rt = pkg("runtime")
    rng = np.random.default_rng(bh * s + d)
    q = rng.standard_normal((bh, s, d)).astype(np.float32)
    k = rng.standard_normal((bh, s, d) if layout == "sd" else (bh, d, s)).astype(np.float32)
    v = rng.standard_normal((bh, s, d)).astype(np.float32)
    o = session.pinned((bh, s, d))
    session.attention_host(pinned_copy(session, q), pinned_copy(session, k), pinned_copy(session, v), o,
                           k_layout=layout)
    session.sync()
    dq, dk, dv = (torch.from_numpy(t).cuda() for t in (q, k, v))
    do = torch.empty_like(dq)
    session.ctx.attention(dq.data_ptr(), dk.data_ptr(), dv.data_ptr(), do.data_ptr(), bh, s, s, d, d,
                          k_layout=rt.K_SD if layout == "sd" else rt.K_DS)
    session.ctx.sync()
    assert np.array_equal(o, do.cpu().numpy())


def test_host_calls_from_pageable_memory(session):
    """Plain NumPy (pageable) buffers: correct, with less overlap."""
    x = np.random.default_rng(9).normal(0, 1, (300, 500)).astype(np.float32)
    y = session.row_softmax_host(x)
    session.sync()
    ref = np.exp(x.astype(np.float64) - x.max(axis=1, keepdims=True))
    ref /= ref.sum(axis=1, keepdims=True)
    np.testing.assert_allclose(y, ref, rtol=1e-5, atol=1e-6)
