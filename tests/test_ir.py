"""The typed Kernel-IR loader: byte-exact round trips of every bundled IR and
rejection of text outside the grammar."""
from __future__ import annotations

import json

import pytest

from conftest import GOLDEN, pkg

IR_FILES = sorted((GOLDEN / "cases").glob("*/*.ir.json"))


def test_bundled_ir_count():
    assert len(IR_FILES) >= 100


@pytest.mark.parametrize("path", IR_FILES, ids=lambda p: p.parent.name)
def test_round_trip_byte_exact(path):
    ir = pkg("ir")
    data = json.loads(path.read_text())
    graph = ir.Graph.from_dict(data)
    assert graph.to_dict() == data
    for kernel in graph.kernels():
        for stmt in kernel.body:
            assert ir.parse(ir.render(stmt)) == stmt


@pytest.mark.parametrize("text", [
    "__import__('os').system('true')",
    "Tile(axes=(), body=(), x=open('/etc/passwd'))",
    "Tile(axes=(), body=[i for i in range(3)])",
    "lambda: 0",
    "Var(name='a').__class__",
    "Foo(x=1)",
    "Var(name='a')",          # an expression, not a statement
])
def test_rejects_non_grammar(text):
    ir = pkg("ir")
    with pytest.raises(ir.IRError):
        ir.parse(text)


def test_field_access_and_walk():
    ir = pkg("ir")
    path = next(p for p in IR_FILES if p.parent.name.startswith("f02_row_softmax"))
    graph = ir.Graph.load(path)
    (kernel,) = graph.kernels()
    tile = kernel.body[0]
    assert tile.kind == "Tile" and tile.block_threads == 128
    assert [a.name for a in tile.axes] == ["a0", "a1_co"]
    assert ir.static_int(tile.axes[0].extent) == 64
    kinds = {s.kind for s in ir.walk(kernel.body)}
    assert {"StridedLoop", "WarpShuffle", "TreeHalve", "Accum", "Write"} <= kinds
