"""BASELINE-sized Kernel-IR cases for the front-end tests (CPU and GPU).

The published IRs (bundled under tests/golden/cases) are rescaled to the
benchmark configurations with ``workloads.scaled_case`` -- the reference's
own recipe, tests/performance/generators/suite.py:313-393 -- and the ragged
configuration is the generated matmul-2 case rewritten with the bias + ReLU
epilogue and a transposed B, then rescaled.
"""
from __future__ import annotations

import json
import math
from pathlib import Path

from conftest import GOLDEN, pkg

CASES = GOLDEN / "cases"
F32 = "DataType(name='f32', np=dtype('float32'), nbytes=4)"

# (family, published template, BASELINE shape, recognised kind)
BASELINE = [
    ("add", "p01_vector_add-5e973341ada3", (1 << 24,), "pointwise"),
    ("softmax", "f02_row_softmax-89d56c168a0b", (4096, 8192), "row_softmax"),
    ("gemm", "m01_matmul_512-cd9a29496fcc", (4096, 4096, 4096), "matmul"),
    ("attention", "a01_attention-c10866af73f8", (2048, 128), "attention"),
]


def scaled(out: Path, family: str, template: str, shape) -> Path:
    return pkg("workloads").scaled_case(CASES / template, out / family, family, shape)


def ragged_case(out: Path, m: int = 4097, n: int = 1000, k: int = 777) -> Path:
    """relu(x @ y^T + bias): matmul-2 (a Tile over (row, col), a K loop over
    kk) with y loaded at (col, kk) from a [n, k] buffer, a bias[n] load and a
    ReLU before the Write, rescaled to m x n x k (block 256, grid covering
    the m * n cells)."""
    src = CASES / "matmul-2-cc1c8cef5b4d"
    graph = json.loads(next(src.glob("*.ir.json")).read_text())
    meta = json.loads((src / "meta.json").read_text())
    node = graph["nodes"]["out_511255"]
    body = node["op_fields"]["body"][0]
    edits = [
        ("input='y_637842', index=(Var(name='kk'), Var(name='col'))",
         "input='y_637842', index=(Var(name='col'), Var(name='kk'))"),
        ("Write(output='out_511255', index=(Var(name='row'), Var(name='col')), values=('total',)",
         f"Load(names=('bv',), input='bias_1', index=(Var(name='col'),), dtype={F32}), "
         f"Assign(name='biased', op=ElementwiseImpl('add'), args=('total', 'bv'), dtype={F32}), "
         f"Assign(name='act', op=ElementwiseImpl('relu'), args=('biased',), dtype={F32}), "
         "Write(output='out_511255', index=(Var(name='row'), Var(name='col')), values=('act',)"),
    ]
    for old, new in edits:
        assert old in body
        body = body.replace(old, new)
    node["op_fields"]["body"][0] = body
    node["inputs"].append("bias_1")
    graph["inputs"].append("bias_1")
    graph["nodes"]["bias_1"] = {"inputs": [], "op": "InputOp", "op_fields": {},
                                "outputs": [{"dtype": "f32", "name": "bias_1", "shape": [n]}]}
    wl = pkg("workloads")
    shapes = {"x_786334": (m, k), "y_637842": (n, k), "out_511255": (m, n), "bias_1": (n,)}
    graph = wl.rescale_graph(graph, shapes, {"row": m, "col": n, "kk": k})
    kernel = meta["kernels"][0]
    kernel["arg_order"].insert(1, "bias_1")
    kernel["args"].append({"dtype": "f32", "name": "bias_1", "shape": [n]})
    meta["graph_inputs"].append("bias_1")
    for i, arg in enumerate(kernel["args"]):
        arg["shape"] = list(shapes[arg["name"]])
        if not arg.get("output"):
            arg["seed"] = 4001 + i
    kernel["grid"] = [math.ceil(m * n / 256), 1, 1]
    folder = out / "ragged"
    folder.mkdir(parents=True, exist_ok=True)
    (folder / "meta.json").write_text(json.dumps(meta))
    path = folder / f"{kernel['entry']}.ir.json"
    path.write_text(json.dumps(graph))
    return path
