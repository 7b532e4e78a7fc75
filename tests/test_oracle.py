"""Pins the CPU oracle: against the reference's own 3xTF32 model outputs and
against every bundled expected output of the hot-path families."""
from __future__ import annotations

import json

import numpy as np
import pytest

from conftest import GOLDEN, golden_cases
from oracle import refs, sexp, tf32


@pytest.fixture(scope="module")
def vectors():
    with np.load(GOLDEN / "tf32" / "vectors.npz") as data:
        return {k: data[k] for k in data.files}


def test_tf32_rna_bit_exact(vectors):
    got = tf32.tf32_rna(vectors["rna_in"]).view(np.uint32)
    want = vectors["rna_out"].view(np.uint32)
    nan = np.isnan(vectors["rna_out"])
    assert np.array_equal(np.isnan(tf32.tf32_rna(vectors["rna_in"])), nan)
    np.testing.assert_array_equal(got[~nan], want[~nan])


def test_simulate_atom_bit_exact(vectors):
    np.testing.assert_array_equal(tf32.simulate(vectors["atom_a"], vectors["atom_b"]), vectors["atom_c"])


@pytest.mark.parametrize("name", ["mm", "wide"])
def test_simulate_matmul_bit_exact(vectors, name):
    got = tf32.simulate_matmul(vectors[f"{name}_a"], vectors[f"{name}_b"])
    np.testing.assert_array_equal(got, vectors[f"{name}_c"])


def test_reference_atom_ptx_fixture_is_pinned():
    """The reference's one-atom PTX (tf32_emitter.synthetic_ptx output, run on
    the GPU by test_gpu_reference_ptx.py) is the file its generator recorded:
    checked by hash only, the text is not inspected."""
    import hashlib
    record = json.loads((GOLDEN / "manifest.json").read_text())["reference_ptx"]
    data = (GOLDEN / record["file"]).read_bytes()
    assert hashlib.sha256(data).hexdigest() == record["sha256"]
    assert record["entry"] == "synthetic_mma"


def test_maxfinite_witness_model_is_nan(vectors):
    """The reference model turns max-finite x 0 into NaN (rna overflows to inf);
    the device split clamps instead, matching the bundled expected 0."""
    with np.errstate(invalid="ignore"):
        got = tf32.simulate(vectors["witness_a"], vectors["witness_b"])
    assert np.isnan(got).all() and np.isnan(vectors["witness_c"]).all()


def test_3xtf32_contract_accuracy():
    rng = np.random.default_rng(5)
    a = rng.uniform(-1, 1, (64, 512)).astype(np.float32)
    b = rng.uniform(-1, 1, (512, 48)).astype(np.float32)
    exact = a.astype(np.float64) @ b.astype(np.float64)
    assert tf32.normwise_error(tf32.gemm_3xtf32(a, b), exact) < 2e-7
    assert tf32.normwise_error(tf32.simulate_matmul(a, b), exact) < 1e-6


def test_selective_exp_model_within_bound():
    x = np.linspace(-110, 10, 200001, dtype=np.float32)
    assert sexp.check_against_exp(x, sexp.model(x))["ok"]
    # the subnormal range survives (FTZ-only would flush these to zero)
    sub = (x > -103.0) & (x < -88.0)
    assert np.all(sexp.model(x)[sub] > 0)


def _meta_data(case_dir, name):
    meta = json.loads((case_dir / "meta.json").read_text())
    for kernel in meta["kernels"]:
        for arg in kernel["args"]:
            if arg["name"] == name and "data" in arg:
                return np.asarray(arg["data"], dtype=np.float32)
    return None


def published_reference(problem, x, case_dir):
    if problem in ("p00_scalar_add", "p01_vector_add"):
        return {"add": refs.pointwise("add", x["x0"], x["x1"])}
    if problem == "p02_scale_shift":
        return {"add": refs.pointwise("scale_shift", x["x"], _meta_data(case_dir, "mul_c1"),
                                      _meta_data(case_dir, "add_c1"))}
    if problem == "p03_relu_mul":
        return {"mul": refs.pointwise("relu_mul", x["x"], x["y"])}
    if problem in ("r01_array_sum", "r02_big_sum"):
        return {"sum_1": refs.array_sum(x["x"])}
    if problem == "r03_mean":
        return {"mean": refs.mean(x["x"])}
    if problem == "r04_row_sum":
        return {"sum_1": refs.row_sum(x["x"])}
    if problem == "f01_rmsnorm":
        return {"mul_1": refs.rmsnorm(x["x"], x["w"], float(_meta_data(case_dir, "add_c1")[0]))}
    if problem == "f02_row_softmax":
        return {"softmax": refs.softmax(x["x"])}
    if problem == "f03_l2norm":
        return {"div": refs.l2norm(x["x"])}
    if problem in ("m01_matmul_512", "m02_matmul_rect"):
        return {"matmul": refs.matmul(x["x0"], x["x1"])}
    if problem in ("a01_attention", "a02_attention_128"):
        return {"matmul_1": refs.attention(x["q"], x["kt"], x["v"], float(x["div_c1"][0]))}
    raise KeyError(problem)


def generated_reference(spec, x):
    """tools/research_cases.py:74-103, keyed by the case's name map."""
    names = spec["names"]
    fam = spec["family"]
    get = lambda k: x[names[k]]
    if fam == "pointwise":
        op = spec["operation"]
        if op == "scale_shift":
            return refs.pointwise("scale_shift", get("x"), get("scale"), get("shift"))
        return refs.pointwise(op, get("x"), get("y"))
    if fam == "reduction":
        return refs.array_sum(get("x"))
    if fam in ("matmul", "atomic_matmul"):
        return refs.matmul(get("x"), get("y"))
    if fam == "softmax":
        return refs.softmax(get("x"))
    if fam == "attention":
        return refs.attention(get("x"), get("y"), get("v"), float(get("scale")[0]))
    if fam == "rmsnorm":
        return refs.rmsnorm(get("x"), None, spec["epsilon"])
    if fam == "l2norm":
        return refs.l2norm(get("x"), spec["epsilon"])
    raise KeyError(fam)


def pinned_cases():
    rows = []
    for case in golden_cases():
        spec = json.loads((GOLDEN / "cases" / case["dir"] / "case.json").read_text()).get("spec", {})
        if spec.get("family") == "published":
            rows.append(pytest.param(case["dir"], id=case["dir"]))
        elif spec.get("version") == "emmy-research-cases-scalar-flatindex-v3" or spec.get("family") == "softmax":
            rows.append(pytest.param(case["dir"], id=case["dir"]))
    return rows


@pytest.mark.parametrize("case_dir", pinned_cases())
def test_refs_reproduce_bundled_expected(case_dir):
    folder = GOLDEN / "cases" / case_dir
    case = json.loads((folder / "case.json").read_text())
    spec = case.get("spec", {})
    meta = json.loads((folder / "meta.json").read_text())
    with np.load(folder / "inputs.npz") as data:
        x = {k: data[k] for k in data.files}
    with np.load(folder / "expected.npz") as data:
        expected = {k: data[k] for k in data.files}
    if spec.get("family") == "published":
        got = published_reference(spec["problem"], x, folder)
    elif "names" in spec and spec.get("version") == "emmy-research-cases-scalar-flatindex-v3":
        got = {spec["names"]["out"]: generated_reference(spec, x)}
    else:  # softmax witnesses keyed by their graph output
        got = {meta["graph_outputs"][0]: refs.softmax(x[spec["names"]["x"]])}
    for name, want in expected.items():
        # same float64 equations, possibly a different summation order: a
        # few FP32 ulps at most, well inside every metadata tolerance
        ok, bad, err = refs.allclose_report(got[name].reshape(want.shape), want, 1e-5, 1e-6)
        assert ok, (name, bad, err)
