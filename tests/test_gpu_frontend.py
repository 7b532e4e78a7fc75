"""Drop-in parity: every recognised bundled case runs through the front end and
the C ABI on the GPU and matches the reference's expected outputs at the
case's own metadata tolerance (tools/research_gpu.py:71-86 comparison)."""
from __future__ import annotations

import json

import numpy as np
import pytest

from conftest import GOLDEN, pkg
from oracle import refs
from test_frontend import RECOGNISED

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def session(ctx):
    api = pkg("api")
    s = api.Session(0)
    yield s
    s.close()


CASES = sorted(n for n, kinds in RECOGNISED.items() if all(kinds) and (GOLDEN / "cases" / n / "expected.npz").exists())


@pytest.mark.parametrize("name", CASES)
def test_recognised_case_matches_expected(session, name):
    runner = pkg("runner")
    folder = GOLDEN / "cases" / name
    meta = json.loads((folder / "meta.json").read_text())
    with np.load(folder / "inputs.npz") as data:
        inputs = {k: data[k] for k in data.files}
    with np.load(folder / "expected.npz") as data:
        expected = {k: data[k] for k in data.files}
    pipeline = runner.Pipeline(folder)
    if any(s.kind == "attention" for s in pipeline.specs) and not hasattr(session.ctx, "attention"):
        pytest.skip("attention kernel not built")
    result, arrays = pipeline.run(session, inputs=inputs, warmup=1, iters=2)
    assert result["ok"]
    for out, want in expected.items():
        ok, bad, err = refs.allclose_report(arrays[out].reshape(want.shape), want, meta["rtol"], meta["atol"])
        assert ok, (out, bad, err)


def test_runner_seeded_request(session):
    """The runner's own seeded-input path (no fixture payload)."""
    runner = pkg("runner")
    result = runner.Pipeline(GOLDEN / "cases" / "p01_vector_add-5e973341ada3").run(session, warmup=1, iters=3)[0]
    x0 = np.random.default_rng(0).standard_normal(1024).astype(np.float32)
    x1 = np.random.default_rng(1).standard_normal(1024).astype(np.float32)
    assert result["outputs"]["add"]["values"] == (x0 + x1).tolist()
    assert result["median_us"] is not None and result["median_us"] > 0


def test_transposed_operand_matmul_runs(session, tmp_path):
    """A recognised x @ y^T (y stored [n, k]) through the runner on the GPU
    against float64 at the matmul tolerance."""
    from test_frontend import transposed_matmul_case
    runner = pkg("runner")
    folder, _ = transposed_matmul_case(tmp_path)
    rng = np.random.default_rng(3)
    x = rng.standard_normal((3, 31)).astype(np.float32)
    y = rng.standard_normal((16, 31)).astype(np.float32)
    result, arrays = runner.Pipeline(folder).run(session, inputs={"x_786334": x, "y_637842": y}, warmup=1, iters=2)
    assert result["ok"] and result["kernels"] == ["matmul"]
    want = x.astype(np.float64) @ y.astype(np.float64).T
    ok, bad, err = refs.allclose_report(arrays["out_511255"].reshape(3, 16), want.astype(np.float32), 1e-3, 1e-3)
    assert ok, (bad, err)


@pytest.mark.parametrize("relu", [True, False])
def test_bias_relu_matmul_runs(session, tmp_path, relu):
    """A recognised relu(x @ y + bias) IR through the runner on the GPU."""
    from test_frontend import bias_relu_matmul_case
    runner = pkg("runner")
    folder, _ = bias_relu_matmul_case(tmp_path, relu)
    rng = np.random.default_rng(4)
    x = rng.standard_normal((3, 31)).astype(np.float32)
    y = rng.standard_normal((31, 16)).astype(np.float32)
    bias = rng.standard_normal(16).astype(np.float32)
    result, arrays = runner.Pipeline(folder).run(session, inputs={"x_786334": x, "y_637842": y, "bias_1": bias},
                                                 warmup=1, iters=2)
    assert result["ok"]
    want = x.astype(np.float64) @ y.astype(np.float64) + bias
    want = np.maximum(want, 0.0) if relu else want
    ok, bad, err = refs.allclose_report(arrays["out_511255"].reshape(3, 16), want.astype(np.float32), 1e-3, 1e-3)
    assert ok, (bad, err)


def test_batched_matmul_runs(session, tmp_path):
    """A recognised batched contraction (x [2, 3, 31] @ y [2, 31, 16]) through the runner."""
    from test_frontend import batched_matmul_case
    runner = pkg("runner")
    folder, _ = batched_matmul_case(tmp_path)
    rng = np.random.default_rng(5)
    x = rng.standard_normal((2, 3, 31)).astype(np.float32)
    y = rng.standard_normal((2, 31, 16)).astype(np.float32)
    result, arrays = runner.Pipeline(folder).run(session, inputs={"x_786334": x, "y_637842": y}, warmup=1, iters=2)
    assert result["ok"]
    want = np.einsum("bmk,bkn->bmn", x.astype(np.float64), y.astype(np.float64))
    ok, bad, err = refs.allclose_report(arrays["out_511255"].reshape(2, 3, 16), want.astype(np.float32), 1e-3, 1e-3)
    assert ok, (bad, err)


def test_transposed_left_operand_matmul_runs(session, tmp_path):
    from test_frontend import transposed_a_matmul_case
    runner = pkg("runner")
    folder, _ = transposed_a_matmul_case(tmp_path)
    rng = np.random.default_rng(6)
    x = rng.standard_normal((31, 3)).astype(np.float32)
    y = rng.standard_normal((31, 16)).astype(np.float32)
    result, arrays = runner.Pipeline(folder).run(session, inputs={"x_786334": x, "y_637842": y}, warmup=1, iters=2)
    assert result["ok"]
    want = x.astype(np.float64).T @ y.astype(np.float64)
    ok, bad, err = refs.allclose_report(arrays["out_511255"].reshape(3, 16), want.astype(np.float32), 1e-3, 1e-3)
    assert ok, (bad, err)
