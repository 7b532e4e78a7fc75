"""The front end on BASELINE-sized Kernel IR, and its exact-once placement
proof on grids far above the sampled-execution budget (CPU).

The published IRs rescaled to the benchmark configurations (tests/
scaled_cases.py, after tests/performance/generators/suite.py:313-393) must be
recognised as the family the benchmark runs, with the output placement
proven for every CTA of the launch and the values certified on two seeds.
A kernel that skips one CTA's tile, or redirects one CTA's writes, on grids
of 8192 and 512 CTAs -- where only a handful of CTAs are executed for values
-- must be refused, and so must a kernel whose write placement depends on data
(the property tensor_core.py:1577-1612 proves by enumerating the launch).
"""
from __future__ import annotations

import json

import pytest

from conftest import pkg
from scaled_cases import BASELINE, ragged_case, scaled


@pytest.mark.parametrize("family,template,shape,kind", BASELINE)
def test_baseline_ir_is_recognised(tmp_path, family, template, shape, kind):
    spec = pkg("frontend").compile_path(scaled(tmp_path, family, template, shape))
    assert spec.kind == kind
    cert = spec.certificate
    assert not cert["exhaustive"] and cert["seeds"] == 2 and "exactly once" in cert["placement"]
    p = spec.params
    if family == "add":
        assert p["n"] == shape[0] and p["insns"][0][0] == "add"
    elif family == "softmax":
        assert (p["rows"], p["cols"]) == shape
    elif family == "gemm":
        assert (p["m"], p["n"], p["k"], p["b_nk"], p["a_t"]) == (*shape, False, False)
    else:
        assert (p["s_q"], p["s_kv"], p["d"], p["dv"]) == (shape[0], shape[0], shape[1], shape[1])


def test_ragged_ir_is_recognised(tmp_path):
    spec = pkg("frontend").compile_path(ragged_case(tmp_path))
    p = spec.params
    assert spec.kind == "matmul"
    assert (p["m"], p["n"], p["k"], p["b_nk"], p["bias"], p["relu"]) == (4097, 1000, 777, True, "bias_1", True)
    assert "exactly once" in spec.certificate["placement"]


# --------------------------------------------------------------------------- tampered placement
WRITE = "Write(output='add', index=(BinaryExpr(op='+', left=BinaryExpr(op='*', left=Var(name='a0'), " \
        "right=Literal(value=2, dtype='int')), right=Literal(value=0, dtype='int')),), values=('v0__u0', 'v0__u1')"
CLOSE = ", value_dtype=DataType(name='f32', np=dtype('float32'), nbytes=4), atomic=False, swizzle='NONE')"


def _bid_is(value: int, op: str = "==") -> str:
    return f"BinaryExpr(op='{op}', left=Builtin(name='block_idx.x'), right=Literal(value={value}, dtype='int'))"


def _tampered(tmp_path, replace):
    """p01_vector_add at n = 2^22 (8192 CTAs of 256 threads, far above the
    execution budget) with its Write statement rewritten by `replace`."""
    path = scaled(tmp_path, "add", "p01_vector_add-5e973341ada3", (1 << 22,))
    graph = json.loads(path.read_text())
    node = graph["nodes"]["add"]
    body = node["op_fields"]["body"][0]
    assert WRITE + CLOSE in body
    node["op_fields"]["body"][0] = body.replace(WRITE + CLOSE, replace(WRITE + CLOSE))
    path.write_text(json.dumps(graph))
    return path


def test_untampered_large_grid_is_accepted(tmp_path):
    spec = pkg("frontend").compile_path(_tampered(tmp_path, lambda w: w))
    assert spec.kind == "pointwise" and spec.certificate["grid"] == 8192
    assert spec.certificate["ctas_executed"] < 16


def test_skipped_cta_tile_is_refused(tmp_path):
    """CTA 5000 of 8192 writes nothing: its 512 outputs are never written."""
    fe = pkg("frontend")
    path = _tampered(tmp_path, lambda w: f"Cond(cond={_bid_is(5000, '!=')}, body=({w},), else_body=())")
    with pytest.raises(fe.Unsupported, match="unwritten"):
        fe.compile_path(path)


def test_redirected_cta_writes_are_refused(tmp_path):
    """m01 at 1024 x 1024 x 512 (512 CTAs of 512 threads, four executed for
    values): CTA 100 writes its first output row one row down, onto the row
    its second Write covers -- one row written twice, one never."""
    fe = pkg("frontend")
    path = scaled(tmp_path, "gemm", "m01_matmul_512-cd9a29496fcc", (1024, 1024, 512))
    graph = json.loads(path.read_text())
    node = graph["nodes"]["matmul"]
    body = node["op_fields"]["body"][0]
    start = body.index("Write(output='matmul'")
    end = body.index("swizzle='NONE')", start) + len("swizzle='NONE')")
    write = body[start:end]
    row0 = "Var(name='a0_u'), right=Literal(value=2, dtype='int'))), right=Literal(value=0, dtype='int'))"
    assert write.count(row0) == 1
    moved = write.replace(row0, row0.replace("value=0", "value=1"))
    guarded = (f"Cond(cond={_bid_is(100)}, body=({moved},), else_body=()), "
               f"Cond(cond={_bid_is(100, '!=')}, body=({write},), else_body=())")
    node["op_fields"]["body"][0] = body[:start] + guarded + body[end:]
    path.write_text(json.dumps(graph))
    with pytest.raises(fe.Unsupported, match="unwritten|more than once"):
        fe.compile_path(path)


def test_data_dependent_placement_is_refused(tmp_path):
    """A Write guarded by a loaded value has no index-only coverage proof."""
    fe = pkg("frontend")
    guard = "BinaryExpr(op='<', left=Var(name='in0__u0'), right=Literal(value=3.0, dtype='float'))"
    path = _tampered(tmp_path, lambda w: f"Cond(cond={guard}, body=({w},), else_body=())")
    with pytest.raises(fe.Unsupported, match="index-only proof"):
        fe.compile_path(path)
