"""The front end (compile_path contract, recogniser) on the bundled fixtures, CPU only."""
from __future__ import annotations

import json
import shutil

import pytest

from conftest import GOLDEN, pkg

CASES = GOLDEN / "cases"

# Recognised hot-path kernels among the bundled fixtures (kernel kinds in
# metadata order; None = outside the recognised families).
RECOGNISED = {
    "a01_attention-c10866af73f8": ["attention"],
    "a02_attention_128-69db4e7f597c": ["attention"],
    "atomic_matmul-0-b0bb43becf74": ["matmul"],
    "atomic_matmul_7x5x9-variant": ["matmul"],
    "attention-0-9170e7b0641d": ["matmul", "row_softmax", "matmul"],
    "canonical-tail-1575656197e9": ["axis_reduce"],
    "canonical-tail-c37693f91a72": ["axis_reduce"],
    "nondivisible-counter-21171f5ca6c3": ["axis_reduce"],
    "short-ring-7bb9d9c27732": ["axis_reduce"],
    "short-ring-b8c0079b7d44": ["axis_reduce"],
    "case-08-e4ac354528a2": ["row_reduce"],
    "case-14-fff293a2235c": ["row_reduce"],
    "case-22-da018f96fc2e": ["row_reduce"],
    "case-30-061d7084b729": ["row_reduce"],
    "case-4-b24c76efd4ba": ["pointwise"],
    "case-7-72f1deeac451": ["matmul"],
    "f01_rmsnorm-6ab09ab4acc3": ["row_norm"],
    "f02-extra-cta-120bf007fb2d": ["row_softmax"],
    "f03_l2norm-1e82d7e58a53": ["row_norm"],
    "l2norm-0-e8f4437dd934": ["row_norm"],
    "r01_array_sum-2ffefe7fee88": ["row_reduce"],
    "r02_big_sum-a56bdb784a46": ["row_reduce"],
    "r03_mean-6dfbe2bc925e": ["row_reduce"],
    "r04_row_sum-5c2ba872d36e": ["row_reduce"],
    "rmsnorm-0-09d6470c83d3": ["row_norm"],
    "f02_row_softmax-89d56c168a0b": ["row_softmax"],
    "full-segment16-274cb67281df": ["attention"],
    "full-segment16-44c6e3443740": ["attention"],
    "full-segment16-899690420377": ["attention"],
    "full-segment16-c974ec730c3e": ["attention"],
    "full-segment16-dd375967ea38": ["attention"],
    "full-segment32-aa23bbd00f94": ["attention"],
    "m01_matmul_512-cd9a29496fcc": ["matmul"],
    "m02_matmul_rect-aeb1568894b7": ["matmul"],
    "matmul-2-cc1c8cef5b4d": ["matmul"],
    "maxfinite-times-zero-v2-991d11340dcd": ["matmul"],
    "p00_scalar_add-4035b0c01010": ["pointwise"],
    "p01_vector_add-5e973341ada3": ["pointwise"],
    "p02_scale_shift-3145aa57f753": ["pointwise"],
    "p03_relu_mul-aeeffce3a36b": ["pointwise"],
    "partial-fallback-bdd094ff243f": ["attention"],
    "partial-fallback-ef3488d3d03c": ["attention"],
    "pointwise-1-fe256034fe7c": ["pointwise"],
    "pointwise-3-06a6f12448fb": ["pointwise"],
    "root-axis-alpha-rename-tid-d51e9f76fb9d": ["attention"],
    "scaled_score_mutable_alias-variant": ["attention"],
    "softmax-0-5200ccc23b31": ["row_softmax"],
    "softmax-1-0a50249d1218": ["row_softmax"],
    "softmax-2-d7aa0ab891e7": ["row_softmax"],
    "tail32-de25e54114aa": ["attention"],
}


def kinds_of(folder):
    fe = pkg("frontend")
    meta = json.loads((folder / "meta.json").read_text())
    irs = sorted(folder.glob("*.ir.json"))
    kinds = []
    for kernel in meta["kernels"]:
        path = folder / f"{kernel['entry']}.ir.json"
        if not path.exists():
            path = irs[0]
        try:
            kinds.append(fe.compile_path(path).kind)
        except fe.Unsupported:
            kinds.append(None)
    return kinds


@pytest.mark.parametrize("name", sorted(p.name for p in CASES.iterdir() if p.is_dir()))
def test_recognition_over_bundled_cases(name):
    kinds = kinds_of(CASES / name)
    assert kinds == RECOGNISED.get(name, [None] * len(kinds))


def test_pointwise_program_of_p02():
    fe = pkg("frontend")
    spec = fe.compile_path(CASES / "p02_scale_shift-3145aa57f753" / "k_add_pointwise.ir.json")
    p = spec.params
    assert p["inputs"] == ["mul_c1", "add_c1", "x"] and p["broadcast"] == [1, 1, 0]
    assert [i[0] for i in p["insns"]] == ["multiply", "add"] and p["n"] == 4096


def test_matmul_roles_follow_shapes_not_arg_order():
    fe = pkg("frontend")
    spec = fe.compile_path(CASES / "m01_matmul_512-cd9a29496fcc" / "k_matmul_2967be.ir.json")
    assert spec.kind == "matmul" and spec.arg_order == ["x1", "x0", "matmul"]
    assert (spec.params["a"], spec.params["b"]) == ("x0", "x1")
    assert not spec.certificate["exhaustive"] and spec.certificate["ctas_executed"] == 4


def _copy_case(tmp_path, name):
    dst = tmp_path / name
    shutil.copytree(CASES / name, dst)
    return dst


def test_duplicate_argument_names_rejected(tmp_path):
    fe = pkg("frontend")
    case = _copy_case(tmp_path, "p01_vector_add-5e973341ada3")
    meta = json.loads((case / "meta.json").read_text())
    meta["kernels"][0]["arg_order"] = ["x0", "x0", "add"]
    (case / "meta.json").write_text(json.dumps(meta))
    with pytest.raises(fe.Unsupported, match="Duplicate"):
        fe.compile_path(case / "k_add_pointwise.ir.json")


def test_short_grid_rejected(tmp_path):
    fe = pkg("frontend")
    case = _copy_case(tmp_path, "p01_vector_add-5e973341ada3")
    meta = json.loads((case / "meta.json").read_text())
    meta["kernels"][0]["grid"] = [1, 1, 1]
    (case / "meta.json").write_text(json.dumps(meta))
    with pytest.raises(fe.Unsupported, match="grid"):
        fe.compile_path(case / "k_add_pointwise.ir.json")


def test_wrong_semantics_rejected(tmp_path):
    """An add kernel whose IR actually subtracts must not be recognised as add."""
    fe = pkg("frontend")
    case = _copy_case(tmp_path, "p01_vector_add-5e973341ada3")
    path = case / "k_add_pointwise.ir.json"
    path.write_text(path.read_text().replace("ElementwiseImpl('add')", "ElementwiseImpl('subtract')"))
    spec = fe.compile_path(path)  # still a pointwise program ...
    assert [i[0] for i in spec.params["insns"]] == ["subtract"]  # ... of the IR's own op


def test_matmul_over_k_prefix():
    """case-7 contracts only the first 63 of 65 K columns: recognised as
    A[:, :63] @ B[:63, :] read through lda = 65, never as the full A @ B."""
    fe = pkg("frontend")
    spec = fe.compile_path(next((CASES / "case-7-72f1deeac451").glob("*.ir.json")))
    p = spec.params
    assert (spec.kind, p["m"], p["n"], p["k"], p["lda"], p["ldb"]) == ("matmul", 64, 32, 63, 65, 32)


def test_vector_group_windows():
    """case-4 loads 4-wide groups at elements 4c + 1 and 4c + 2 and writes at
    4c: out[i] = x[i + 1] + y[i + 2], two streams with window offsets."""
    fe = pkg("frontend")
    spec = fe.compile_path(next((CASES / "case-4-b24c76efd4ba").glob("*.ir.json")))
    p = spec.params
    assert dict(zip(p["inputs"], p["offsets"])) == {"x_799729": 1, "y_221412": 2}
    assert p["n"] == 260 and p["insns"] == [("add", 1, 0, 0, 0.0)]
    prog = spec.descriptor().program
    assert prog is not None


def transposed_matmul_case(tmp_path):
    """matmul-2 rewritten to read its right operand transposed: y stored
    [16, 31] and loaded at (col, kk), so out = x @ y^T."""
    folder = _copy_case(tmp_path, "matmul-2-cc1c8cef5b4d")
    path = next(folder.glob("*.ir.json"))
    graph = json.loads(path.read_text())
    graph["nodes"]["y_637842"]["outputs"][0]["shape"] = [16, 31]
    body = graph["nodes"]["out_511255"]["op_fields"]["body"][0]
    old = "input='y_637842', index=(Var(name='kk'), Var(name='col'))"
    assert old in body
    graph["nodes"]["out_511255"]["op_fields"]["body"][0] = body.replace(
        old, "input='y_637842', index=(Var(name='col'), Var(name='kk'))")
    path.write_text(json.dumps(graph))
    meta = json.loads((folder / "meta.json").read_text())
    for arg in meta["kernels"][0]["args"]:
        if arg["name"] == "y_637842":
            arg["shape"] = [16, 31]
    (folder / "meta.json").write_text(json.dumps(meta))
    for name in ("inputs.npz", "expected.npz"):
        (folder / name).unlink()
    return folder, path


F32 = "DataType(name='f32', np=dtype('float32'), nbytes=4)"


def bias_relu_matmul_case(tmp_path, relu=True):
    """matmul-2 rewritten with the ragged config's epilogue: out =
    relu(x @ y + bias[col]) (or without the ReLU), bias a [16] input."""
    folder = _copy_case(tmp_path, "matmul-2-cc1c8cef5b4d")
    path = next(folder.glob("*.ir.json"))
    graph = json.loads(path.read_text())
    node = graph["nodes"]["out_511255"]
    body = node["op_fields"]["body"][0]
    write = "Write(output='out_511255', index=(Var(name='row'), Var(name='col')), values=('total',)"
    assert write in body
    epilogue = (f"Load(names=('bv',), input='bias_1', index=(Var(name='col'),), dtype={F32}), "
                f"Assign(name='biased', op=ElementwiseImpl('add'), args=('total', 'bv'), dtype={F32}), ")
    result = "biased"
    if relu:
        epilogue += f"Assign(name='act', op=ElementwiseImpl('relu'), args=('biased',), dtype={F32}), "
        result = "act"
    node["op_fields"]["body"][0] = body.replace(
        write, epilogue + f"Write(output='out_511255', index=(Var(name='row'), Var(name='col')), values=('{result}',)")
    node["inputs"].append("bias_1")
    graph["inputs"].append("bias_1")
    graph["nodes"]["bias_1"] = {"inputs": [], "op": "InputOp", "op_fields": {},
                                "outputs": [{"dtype": "f32", "name": "bias_1", "shape": [16]}]}
    path.write_text(json.dumps(graph))
    meta = json.loads((folder / "meta.json").read_text())
    meta["graph_inputs"].append("bias_1")
    kernel = meta["kernels"][0]
    kernel["arg_order"].insert(1, "bias_1")
    kernel["args"].append({"dtype": "f32", "name": "bias_1", "shape": [16]})
    (folder / "meta.json").write_text(json.dumps(meta))
    for name in ("inputs.npz", "expected.npz"):
        (folder / name).unlink()
    return folder, path


@pytest.mark.parametrize("relu", [True, False])
def test_matmul_bias_relu_epilogue(tmp_path, relu):
    fe = pkg("frontend")
    rt = pkg("runtime")
    _, path = bias_relu_matmul_case(tmp_path, relu)
    spec = fe.compile_path(path)
    p = spec.params
    assert (spec.kind, p["bias"], p["relu"], p["b_nk"]) == ("matmul", "bias_1", relu, False)
    desc = spec.descriptor()
    assert desc.role[3] == spec.arg_order.index("bias_1") and desc.flags[1] == int(relu)


def batched_matmul_case(tmp_path, batch=2):
    """matmul-2 rewritten as a batch of contractions: a third Tile axis `bat`
    indexes x [B, 3, 31], y [B, 31, 16] and out [B, 3, 16]."""
    folder = _copy_case(tmp_path, "matmul-2-cc1c8cef5b4d")
    path = next(folder.glob("*.ir.json"))
    graph = json.loads(path.read_text())
    node = graph["nodes"]["out_511255"]
    body = node["op_fields"]["body"][0]
    for old, new in (
            ("Tile(axes=(Axis(name='row'", f"Tile(axes=(Axis(name='bat', extent=Dim({batch}), window=None), Axis(name='row'"),
            ("input='x_786334', index=(Var(name='row'), Var(name='kk'))",
             "input='x_786334', index=(Var(name='bat'), Var(name='row'), Var(name='kk'))"),
            ("input='y_637842', index=(Var(name='kk'), Var(name='col'))",
             "input='y_637842', index=(Var(name='bat'), Var(name='kk'), Var(name='col'))"),
            ("Write(output='out_511255', index=(Var(name='row'), Var(name='col'))",
             "Write(output='out_511255', index=(Var(name='bat'), Var(name='row'), Var(name='col'))")):
        assert old in body
        body = body.replace(old, new)
    node["op_fields"]["body"][0] = body
    shapes = {"x_786334": [batch, 3, 31], "y_637842": [batch, 31, 16], "out_511255": [batch, 3, 16]}
    for name, shape in shapes.items():
        graph["nodes"][name]["outputs"][0]["shape"] = shape
    path.write_text(json.dumps(graph))
    meta = json.loads((folder / "meta.json").read_text())
    for arg in meta["kernels"][0]["args"]:
        arg["shape"] = shapes[arg["name"]]
    (folder / "meta.json").write_text(json.dumps(meta))
    for name in ("inputs.npz", "expected.npz"):
        (folder / name).unlink()
    return folder, path


def test_batched_matmul(tmp_path):
    fe = pkg("frontend")
    rt = pkg("runtime")
    _, path = batched_matmul_case(tmp_path)
    spec = fe.compile_path(path)
    p = spec.params
    assert (spec.kind, p["batch"], p["m"], p["n"], p["k"], p["b_nk"], p["relu"]) == ("matmul", 2, 3, 16, 31, False,
                                                                                        False)
    desc = spec.descriptor()
    assert desc.kind == rt.KIND_GEMM_BATCHED and tuple(desc.dims[:4]) == (2, 3, 16, 31)


def transposed_a_matmul_case(tmp_path):
    """matmul-2 rewritten to read its left operand transposed: x stored
    [31, 3] and loaded at (kk, row), so out = x^T @ y."""
    folder = _copy_case(tmp_path, "matmul-2-cc1c8cef5b4d")
    path = next(folder.glob("*.ir.json"))
    graph = json.loads(path.read_text())
    graph["nodes"]["x_786334"]["outputs"][0]["shape"] = [31, 3]
    body = graph["nodes"]["out_511255"]["op_fields"]["body"][0]
    old = "input='x_786334', index=(Var(name='row'), Var(name='kk'))"
    assert old in body
    graph["nodes"]["out_511255"]["op_fields"]["body"][0] = body.replace(
        old, "input='x_786334', index=(Var(name='kk'), Var(name='row'))")
    path.write_text(json.dumps(graph))
    meta = json.loads((folder / "meta.json").read_text())
    for arg in meta["kernels"][0]["args"]:
        if arg["name"] == "x_786334":
            arg["shape"] = [31, 3]
    (folder / "meta.json").write_text(json.dumps(meta))
    for name in ("inputs.npz", "expected.npz"):
        (folder / name).unlink()
    return folder, path


def test_matmul_with_transposed_left_operand(tmp_path):
    fe = pkg("frontend")
    rt = pkg("runtime")
    _, path = transposed_a_matmul_case(tmp_path)
    spec = fe.compile_path(path)
    p = spec.params
    assert (spec.kind, p["a"], p["a_t"], p["b_nk"], p["m"], p["n"], p["k"], p["lda"]) == (
        "matmul", "x_786334", True, False, 3, 16, 31, 3)
    desc = spec.descriptor()
    assert desc.flags[0] == rt.A_KM | rt.B_KN and tuple(desc.dims[:6]) == (3, 16, 31, 3, 16, 16)


def test_matmul_with_transposed_operand(tmp_path):
    fe = pkg("frontend")
    rt = pkg("runtime")
    _, path = transposed_matmul_case(tmp_path)
    spec = fe.compile_path(path)
    p = spec.params
    assert (spec.kind, p["a"], p["b"], p["b_nk"], p["m"], p["n"], p["k"], p["ldb"]) == (
        "matmul", "x_786334", "y_637842", True, 3, 16, 31, 31)
    desc = spec.descriptor()
    assert desc.flags[0] == rt.B_NK and tuple(desc.dims[:6]) == (3, 16, 31, 31, 31, 16)


def test_scaled_scores_read_the_divisor_buffer():
    """attention-0's first kernel is scores = x @ y / scale[0]: a GEMM whose
    epilogue divides by the one-element buffer, read at run time."""
    fe = pkg("frontend")
    folder = CASES / "attention-0-9170e7b0641d"
    spec = fe.compile_path(folder / "k_scores_238734.ir.json")
    p = spec.params
    assert (spec.kind, p["a"], p["b"], p["div_buffer"], p["m"], p["n"], p["k"]) == (
        "matmul", "x_992187", "y_390031", "scale_236779", 3, 33, 33)
    desc = spec.descriptor()
    assert desc.role[4] == spec.arg_order.index("scale_236779")


@pytest.mark.parametrize("name, batch, s, cols", [("canonical-tail-1575656197e9", 2, 9, 64),
                                                  ("short-ring-b8c0079b7d44", 3, 1, 64)])
def test_middle_axis_sum(name, batch, s, cols):
    """out[b, j] = sum_i x[b, i, j], whatever ring or counter the IR stages it through."""
    fe = pkg("frontend")
    spec = fe.compile_path(next((CASES / name).glob("*.ir.json")))
    p = spec.params
    assert (spec.kind, p["op"], p["batch"], p["s"], p["cols"], p["sum_div"]) == ("axis_reduce", "sum", batch, s, cols,
                                                                                  1.0)


def test_matmul_prefix_needs_the_certificate(tmp_path):
    """A K guard that is not a prefix (every other column) fits no candidate."""
    fe = pkg("frontend")
    folder = _copy_case(tmp_path, "case-7-72f1deeac451")
    path = next(folder.glob("*.ir.json"))
    text = path.read_text()
    guard = "BinaryExpr(op='<', left=Var(name='kk'), right=Literal(value=63, dtype='int'))"
    assert guard in text
    odd = ("BinaryExpr(op='==', left=BinaryExpr(op='%', left=Var(name='kk'), right=Literal(value=2, dtype='int')), "
           "right=Literal(value=0, dtype='int'))")
    path.write_text(text.replace(guard, odd))
    with pytest.raises(fe.Unsupported):
        fe.compile_path(path)


def test_row_constants_bound_to_metadata_buffers():
    """f01's count and epsilon live in one-element buffers; the kernel must read
    them at run time rather than bake the fitted values."""
    fe = pkg("frontend")
    p = fe.compile_path(CASES / "f01_rmsnorm-6ab09ab4acc3" / "k_mean_cbd1de.ir.json").params
    assert (p["op"], p["w"], p["eps_buffer"], p["count_buffer"]) == ("rmsnorm", "w", "add_c1", "mean_count")
    p = fe.compile_path(CASES / "r03_mean-6dfbe2bc925e" / "k_mean_ffcca3.ir.json").params
    assert (p["sum_div"], p["sum_div_buffer"]) == (32768.0, "mean_keepdim_count")
    p = fe.compile_path(next((CASES / "rmsnorm-0-09d6470c83d3").glob("*.ir.json"))).params
    assert p["eps"] == 1e-05 and p["eps_buffer"] is None


def test_one_value_fit_is_not_enough():
    """A one-output kernel computing 4*x[0] must not pass as a scaled sum."""
    fe = pkg("frontend")
    with pytest.raises(fe.Unsupported):
        fe.compile_path(next((CASES / "axis-rebound-before-load-e5a00bcecf77").glob("*.ir.json")))


def test_cli_contract(capsys):
    fe = pkg("frontend")
    assert fe.main([str(CASES / "p00_scalar_add-4035b0c01010" / "k_add_pointwise.ir.json")]) == 0
    out = json.loads(capsys.readouterr().out)
    assert out["kind"] == "pointwise"
    assert fe.main([str(next((CASES / "case-02-6cbcd2d46537").glob("*.ir.json")))]) == 1
    assert "f16" in capsys.readouterr().err
    assert fe.main([]) == 1
