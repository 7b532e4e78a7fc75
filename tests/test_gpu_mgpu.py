"""GPU tests of the native multi-GPU driver (b2k_mgpu_*, NCCL) through the C ABI.

On one GPU the communicator has one rank: the broadcast of B's panels, the
per-piece gathers, the packing of [K, N] panels and the placement copies all
run, and every result must match the single-GPU entry points (the same
kernels on the same rows) -- bit for bit where the kernel and its tile
choice are the same, else within the 3xTF32 GEMM's normwise bound.  A rank
that never joins ends b2k_mgpu_init with a bounded timeout (made on the
host: the peer simply never calls init).  With two GPUs the same problems
run as two ranks in child processes and gather to the single-GPU results.
NVLS is off in every NCCL communicator these tests create.
"""
from __future__ import annotations

import os
import subprocess
import sys

import numpy as np
import pytest

from conftest import ROOT, pkg
from oracle import tf32

pytestmark = pytest.mark.gpu

os.environ.setdefault("NCCL_NVLS_ENABLE", "0")


def dev(torch, array):
    return torch.from_numpy(np.ascontiguousarray(array)).cuda()


@pytest.fixture(scope="module")
def group(ctx):
    rt = pkg("runtime")
    mg = rt.MultiGpu(ctx, 1, 0, rt.mgpu_unique_id(), timeout_ms=60000)
    yield mg
    mg.close()


@pytest.mark.parametrize("b_layout,panels,bias", [(0, 1, False), (0, 2, True), (0, 3, False), (1, 1, True),
                                                  (1, 2, False)])
def test_world1_gemm_matches_single_gpu(ctx, torch_cuda, group, b_layout, panels, bias):
    torch = torch_cuda
    rng = np.random.default_rng(11 + panels + 5 * b_layout)
    m, n, k = 384, 640, 320
    a = rng.uniform(-1, 1, (m, k)).astype(np.float32)
    b = rng.uniform(-1, 1, (k, n) if b_layout == 0 else (n, k)).astype(np.float32)
    bv = rng.uniform(-0.5, 0.5, n).astype(np.float32) if bias else None
    da, db = dev(torch, a), dev(torch, b)
    dbias = dev(torch, bv) if bias else None
    c_mg = torch.full((m, n), float("nan"), device="cuda")
    group.gemm(da.data_ptr(), db.data_ptr(), c_mg.data_ptr(), m, n, k, b_layout=b_layout,
               bias=dbias.data_ptr() if bias else 0, relu=bias, panels=panels)
    group.sync()
    got = c_mg.cpu().numpy()
    b64 = b.astype(np.float64) if b_layout == 0 else b.astype(np.float64).T
    exact = a.astype(np.float64) @ b64
    if bias:
        exact = np.maximum(exact + bv, 0.0)
    assert np.isfinite(got).all()
    assert tf32.normwise_error(got, exact) <= 1e-5
    # each panel is the single-GPU GEMM of those columns
    cols = [pkg("mgpu").partition(n, panels, p) for p in range(panels)]
    for p in cols:
        sl = slice(p.start, p.start + p.count)
        bp = dev(torch, b[:, sl] if b_layout == 0 else b[sl])
        cp = torch.empty((m, p.count), device="cuda")
        ctx.gemm(da.data_ptr(), bp.data_ptr(), cp.data_ptr(), m, p.count, k, b_layout=b_layout,
                 bias=dbias[sl].data_ptr() if bias else 0, relu=bias)
        ctx.sync()
        np.testing.assert_array_equal(got[:, sl], cp.cpu().numpy())


@pytest.mark.parametrize("pieces", [1, 2, 4])
def test_world1_softmax_pointwise_attention_match_single_gpu(ctx, torch_cuda, group, pieces):
    torch = torch_cuda
    rt = pkg("runtime")
    rng = np.random.default_rng(pieces)
    x = dev(torch, rng.normal(0, 4, (64, 1000)).astype(np.float32))
    y_mg, y = torch.empty_like(x), torch.empty_like(x)
    group.row_softmax(x.data_ptr(), y_mg.data_ptr(), 64, 1000, pieces=pieces)
    ctx.row_softmax(x.data_ptr(), y.data_ptr(), 64, 1000)
    group.sync()
    ctx.sync()
    assert torch.equal(y_mg, y)

    n = 1 << 16
    a, b = (dev(torch, rng.uniform(-1, 1, n).astype(np.float32)) for _ in range(2))
    prog = rt.make_program(2, [("add", 0, 1, 0, 0.0)], 2)
    c_mg, c = torch.empty_like(a), torch.empty_like(a)
    group.pointwise(prog, [a.data_ptr(), b.data_ptr()], c_mg.data_ptr(), n, align=4, pieces=pieces)
    group.sync()
    assert torch.equal(c_mg, a + b)

    bh, s, d = 8, 256, 64
    q, kk, v = (dev(torch, rng.normal(0, 1, (bh, s, d)).astype(np.float32)) for _ in range(3))
    o_mg, o = torch.empty_like(q), torch.empty_like(q)
    group.attention(q.data_ptr(), kk.data_ptr(), v.data_ptr(), o_mg.data_ptr(), bh, s, s, d, d, pieces=pieces)
    ctx.attention(q.data_ptr(), kk.data_ptr(), v.data_ptr(), o.data_ptr(), bh, s, s, d, d)
    group.sync()
    ctx.sync()
    assert torch.equal(o_mg, o)


_NEVER_JOINS = r"""
import os, sys
sys.path.insert(0, sys.argv[1])
os.environ["NCCL_NVLS_ENABLE"] = "0"
import importlib, time
rt = importlib.import_module("emmy-hackathon-2026_b200.runtime")
ctx = rt.Context(0)
t0 = time.time()
try:
    rt.MultiGpu(ctx, 2, 0, rt.mgpu_unique_id(), timeout_ms=3000)
    print("JOINED")
except rt.B2KError as exc:
    print("STATUS", exc.args[0] if exc.args else None, round(time.time() - t0, 2), str(exc)[:200])
ctx.sync()
print("CONTEXT_OK")
"""


def test_rank_that_never_joins_times_out(torch_cuda):
    """World 2, rank 1 never calls init: rank 0's init returns a timeout
    within its bound and the context stays usable (host-side failure; no
    GPU kernel waits on anything)."""
    done = subprocess.run([sys.executable, "-c", _NEVER_JOINS, str(ROOT)], capture_output=True, text=True,
                          timeout=120)
    out = done.stdout
    assert "JOINED" not in out, out + done.stderr
    assert "STATUS" in out, out + done.stderr
    assert "CONTEXT_OK" in out, out + done.stderr


_TWO_RANKS = r"""
import os, sys
root, rank, uid_hex = sys.argv[1], int(sys.argv[2]), sys.argv[3]
sys.path.insert(0, root)
os.environ["NCCL_NVLS_ENABLE"] = "0"
import importlib
import numpy as np
import torch
rt = importlib.import_module("emmy-hackathon-2026_b200.runtime")
mgpu = importlib.import_module("emmy-hackathon-2026_b200.mgpu")
torch.cuda.set_device(rank)
ctx = rt.Context(rank)
group = rt.MultiGpu(ctx, 2, rank, bytes.fromhex(uid_hex), timeout_ms=60000)
rng = np.random.default_rng(5)
m, n, k = 1029, 768, 256                     # uneven row shards: 512 and 517 rows (align 128)
a = rng.uniform(-1, 1, (m, k)).astype(np.float32)
b = rng.uniform(-1, 1, (k, n)).astype(np.float32)
da, db = torch.from_numpy(a).cuda(), torch.from_numpy(b).cuda()
worst = 0.0
for panels in (1, 2):
    sh = mgpu.partition(m, 2, rank, 128)
    c = torch.full((m, n), float("nan"), device="cuda")
    group.gemm(da[sh.start:sh.start + sh.count].contiguous().data_ptr(), db.data_ptr() if rank == 0 else 0,
               c.data_ptr(), m, n, k, align=128, panels=panels)
    group.sync()
    full = torch.empty((m, n), device="cuda")
    ctx.gemm(da.data_ptr(), db.data_ptr(), full.data_ptr(), m, n, k)
    ctx.sync()
    worst = max(worst, float((c - full).abs().max() / full.abs().max()))
rows, cols = 512, 777
x = torch.from_numpy(rng.normal(0, 4, (rows, cols)).astype(np.float32)).cuda()
sh = mgpu.partition(rows, 2, rank)
y = torch.empty_like(x)
group.row_softmax(x[sh.start:sh.start + sh.count].contiguous().data_ptr(), y.data_ptr(), rows, cols, pieces=2)
ref = torch.empty_like(x)
ctx.row_softmax(x.data_ptr(), ref.data_ptr(), rows, cols)
group.sync()
ctx.sync()
exact = bool(torch.equal(y, ref))
group.close()
print("RESULT", rank, worst, exact)
"""


def test_two_ranks_gather_to_single_gpu_results(torch_cuda):
    """Two ranks on two GPUs (skipped with fewer): row-partitioned GEMM with
    uneven shards, whole and in panels, and row softmax in pieces, each
    gathered to the single-GPU result on every rank."""
    if torch_cuda.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    uid = pkg("runtime").mgpu_unique_id().hex()
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    procs = [subprocess.Popen([sys.executable, "-c", _TWO_RANKS, str(ROOT), str(r), uid], stdout=subprocess.PIPE,
                              stderr=subprocess.PIPE, text=True, env=env) for r in range(2)]
    outs = []
    for p in procs:
        try:
            out, err = p.communicate(timeout=240)
        except subprocess.TimeoutExpired:
            p.kill()
            out, err = p.communicate()
        outs.append((p.returncode, out, err))
    for rc, out, err in outs:
        assert rc == 0, out + err[-2000:]
        line = [ln for ln in out.splitlines() if ln.startswith("RESULT")][0].split()
        assert float(line[2]) <= 5e-7, line      # same kernels; a panel may take another tile path
        assert line[3] == "True", line
