"""GPU parity of the batched 3xTF32 attention through the C ABI against the
float64 reference (attention family tolerance: rtol 1e-3, atol 1e-4,
tools/research_cases.py:30-35)."""
from __future__ import annotations

import math

import numpy as np
import pytest

from conftest import pkg
from oracle import refs

pytestmark = pytest.mark.gpu

RTOL, ATOL = 1e-3, 1e-4


def run(ctx, torch, q, k, v, *, k_layout=0, scale=None, scale_buf=None):
    bh, s_q, d = q.shape
    s_kv, dv = v.shape[1], v.shape[2]
    dq, dk, dvv = (torch.from_numpy(np.ascontiguousarray(t)).cuda() for t in (q, k, v))
    do = torch.full((bh, s_q, dv), float("nan"), device="cuda")
    sb = torch.from_numpy(np.asarray([scale_buf], np.float32)).cuda() if scale_buf is not None else None
    ctx.attention(dq.data_ptr(), dk.data_ptr(), dvv.data_ptr(), do.data_ptr(), bh, s_q, s_kv, d, dv,
                  scale=scale, scale_ptr=sb.data_ptr() if sb is not None else 0, k_layout=k_layout)
    ctx.sync()
    return do.cpu().numpy()


@pytest.mark.parametrize("bh,s_q,s_kv,d,dv", [(2, 128, 128, 64, 64), (3, 100, 77, 48, 16), (1, 12, 3, 48, 16),
                                              (4, 256, 512, 128, 128), (1, 9, 19, 19, 7), (2, 200, 300, 32, 40)])
@pytest.mark.parametrize("k_layout", [0, 1])
def test_attention_matches_float64(ctx, torch_cuda, bh, s_q, s_kv, d, dv, k_layout):
    rng = np.random.default_rng(bh * 1000 + s_q + s_kv + d)
    q = rng.standard_normal((bh, s_q, d)).astype(np.float32)
    k = rng.standard_normal((bh, s_kv, d)).astype(np.float32)
    v = rng.standard_normal((bh, s_kv, dv)).astype(np.float32)
    kin = k if k_layout == 0 else np.ascontiguousarray(k.transpose(0, 2, 1))
    got = run(ctx, torch_cuda, q, kin, v, k_layout=k_layout)
    want = refs.attention_batched(q, k, v, math.sqrt(d))
    ok, bad, err = refs.allclose_report(got, want, RTOL, ATOL)
    assert ok, (bad, err)


@pytest.mark.parametrize("bh,s_q,s_kv,d,dv", [(2, 300, 257, 128, 128), (1, 64, 64, 64, 64), (3, 129, 33, 100, 24),
                                         (2, 256, 200, 128, 64), (1, 640, 384, 32, 128)])
def test_attention_paths_agree(ctx, torch_cuda, bh, s_q, s_kv, d, dv):
    """The fused kernel (1, the default) and the three passes (0) against
    float64 and each other."""
    runtime = pkg("runtime")
    lib = runtime.library()
    rng = np.random.default_rng(17 + s_q)
    q = rng.standard_normal((bh, s_q, d)).astype(np.float32)
    k = rng.standard_normal((bh, s_kv, d)).astype(np.float32)
    v = rng.standard_normal((bh, s_kv, dv)).astype(np.float32)
    want = refs.attention_batched(q, k, v, math.sqrt(d))
    outs = []
    try:
        for mode in (1, 0):
            assert lib.b2k_attention_set_fused(mode) == runtime.B2K_OK
            outs.append(run(ctx, torch_cuda, q, k, v))
    finally:
        lib.b2k_attention_set_fused(1)
    for got in outs:
        ok, bad, err = refs.allclose_report(got, want, RTOL, ATOL)
        assert ok, (bad, err)
    np.testing.assert_allclose(outs[0], outs[1], rtol=1e-5, atol=1e-6)
    assert lib.b2k_attention_set_fused(2) == runtime.B2K_EINVAL


def test_attention_scale_from_device_buffer(ctx, torch_cuda):
    """The IR passes the divisor as a one-element buffer (a01's div_c1 = 8)."""
    rng = np.random.default_rng(1)
    q, k, v = (rng.standard_normal((1, 64, 64)).astype(np.float32) for _ in range(3))
    got = run(ctx, torch_cuda, q, k, v, scale_buf=8.0)
    want = refs.attention_batched(q, k, v, 8.0)
    ok, bad, err = refs.allclose_report(got, want, RTOL, ATOL)
    assert ok, (bad, err)


def test_attention_baseline_config_every_head(ctx, torch_cuda):
    """4 x 16 heads, S 2048, D 128: every output of all 64 heads against
    float64 at the attention family's tolerance."""
    workloads = pkg("workloads")
    q, k, v = workloads.attention_inputs()
    got = run(ctx, torch_cuda, q, k, v)
    want = refs.attention_batched(q, k, v, math.sqrt(128))
    ok, bad, err = refs.allclose_report(got, want, RTOL, ATOL)
    assert ok, (bad, err)
