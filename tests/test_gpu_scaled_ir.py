"""BASELINE-sized Kernel IR end to end on the GPU: the published IRs rescaled
to the benchmark configurations (tests/scaled_cases.py) are recognised by
the front end, launched through b2k_launch by the runner's pipeline (seeded
inputs from the scaled metadata, zero_outputs, the positional arg_order
arguments) and compared in full with the reference's float64 equations at
each family's metadata tolerance: pointwise 0 / 0 (bit-exact), softmax
1e-3 / 1e-5, matmul 1e-3 / 1e-3 (and 1e-5 normwise against float64),
attention 1e-3 / 1e-4.  Attention's IR family is one head (q [S, D],
kt [D, S], v [S, D]); the BASELINE configuration is 64 such heads."""
from __future__ import annotations

import math

import numpy as np
import pytest

from conftest import pkg
from oracle import refs, tf32
from scaled_cases import BASELINE, ragged_case, scaled

pytestmark = pytest.mark.gpu


def run_case(path):
    runner, api = pkg("runner"), pkg("api")
    pipeline = runner.Pipeline(path.parent)
    assert len(pipeline.specs) == 1
    inputs = {name: runner.array_for(arg) for name, arg in pipeline.args.items() if not arg.get("output")}
    with api.Session(0) as session:
        result, arrays = pipeline.run(session, inputs=inputs, warmup=0, iters=1, max_return=0)
    assert result["ok"]
    return pipeline, inputs, arrays


@pytest.mark.parametrize("family,template,shape,kind", BASELINE)
def test_baseline_ir_runs_through_b2k_launch(tmp_path, torch_cuda, family, template, shape, kind):
    pipeline, x, out = run_case(scaled(tmp_path, family, template, shape))
    assert pipeline.specs[0].kind == kind
    if family == "add":
        np.testing.assert_array_equal(out["add"], refs.pointwise("add", x["x0"], x["x1"]))
    elif family == "softmax":
        ok, bad, err = refs.allclose_report(out["softmax"], refs.softmax(x["x"]), 1e-3, 1e-5)
        assert ok, (bad, err)
    elif family == "gemm":
        exact = x["x0"].astype(np.float64) @ x["x1"].astype(np.float64)
        assert tf32.normwise_error(out["matmul"], exact) <= 1e-5
        ok, bad, err = refs.allclose_report(out["matmul"], exact.astype(np.float32), 1e-3, 1e-3)
        assert ok, (bad, err)
    else:
        want = refs.attention(x["q"], x["kt"], x["v"], math.sqrt(shape[1]))
        ok, bad, err = refs.allclose_report(out["matmul_1"], want, 1e-3, 1e-4)
        assert ok, (bad, err)


def test_ragged_ir_runs_through_b2k_launch(tmp_path, torch_cuda):
    pipeline, x, out = run_case(ragged_case(tmp_path))
    want = refs.matmul_bias_relu(x["x_786334"], x["y_637842"], x["bias_1"])
    ok, bad, err = refs.allclose_report(out["out_511255"], want, 1e-3, 1e-3)
    assert ok, (bad, err)
