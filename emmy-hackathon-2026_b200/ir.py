"""Typed Emmy Kernel-IR: a safe loader for the ``*.ir.json`` graph format.

The reference compiler loads kernels with the third-party ``emmy-ml==0.3.11``
package (``Graph.from_dict``, called at compile.py:9630; the statement classes
are imported at compile.py:15-16 and tensor_core.py:15-20).  That package is
not part of this backend.  The on-disk format is plain JSON whose
``KernelOp.op_fields.body`` entries are Python ``repr`` strings of statement
constructors, e.g. ``Tile(axes=(Axis(name='a0', extent=Dim(64), window=None),),
body=(...))``.  This module parses those strings with :mod:`ast` -- never with
``eval`` -- accepting only the constructor vocabulary of the format, and
renders them back byte-identically, so a loaded graph round-trips to the exact
JSON it came from.

Nodes keep the constructor name in ``kind`` and the fields in declaration
order; fields are read as attributes (``stmt.body``, ``expr.left``).
"""
from __future__ import annotations

import ast
import json
from pathlib import Path
from typing import Any, Iterable, Iterator

# Constructor vocabulary of the serialised statement/expression language, with
# the names of fields that the format writes positionally (``Dim(64)``,
# ``ElementwiseImpl('add')``, ``dtype('float32')``).
CONSTRUCTORS: dict[str, tuple[str, ...]] = {
    # statements
    "Tile": (), "Loop": (), "StridedLoop": (), "Load": (), "Write": (), "Assign": (),
    "Let": (), "Accum": (), "Init": (), "Cond": (), "Select": (), "SelectBranch": (),
    "Smem": (), "Sync": (), "WarpShuffle": (), "TreeHalve": (), "CpAsyncCopy": (),
    "CpAsyncCommit": (), "CpAsyncWait": (),
    # axes and types
    "Axis": (), "Dim": ("value",), "Window": (), "DataType": (), "dtype": ("name",),
    "ElementwiseImpl": ("name",),
    # expressions
    "BinaryExpr": (), "TernaryExpr": (), "Literal": (), "Var": (), "Builtin": (),
    "FuncCallExpr": (), "CastExpr": (), "FlatIndex": (),
}

STATEMENTS = frozenset({
    "Tile", "Loop", "StridedLoop", "Load", "Write", "Assign", "Let", "Accum", "Init",
    "Cond", "Select", "SelectBranch", "Smem", "Sync", "WarpShuffle", "TreeHalve",
    "CpAsyncCopy", "CpAsyncCommit", "CpAsyncWait",
})

MAX_SOURCE = 8_000_000  # bytes of one body string


class IRError(ValueError):
    """The IR text is outside the accepted Kernel-IR grammar."""


class Node:
    """One constructor application: ``kind(*positional, **fields)``."""

    __slots__ = ("kind", "positional", "fields")

    def __init__(self, kind: str, positional: tuple = (), fields: dict | None = None):
        self.kind = kind
        self.positional = tuple(positional)
        self.fields = dict(fields or {})

    def __getattr__(self, name: str) -> Any:
        if name.startswith("__"):
            raise AttributeError(name)
        fields = object.__getattribute__(self, "fields")
        if name in fields:
            return fields[name]
        names = CONSTRUCTORS.get(object.__getattribute__(self, "kind"), ())
        positional = object.__getattribute__(self, "positional")
        if name in names and names.index(name) < len(positional):
            return positional[names.index(name)]
        raise AttributeError(f"{self.kind} has no field {name!r}")

    def get(self, name: str, default: Any = None) -> Any:
        try:
            return getattr(self, name)
        except AttributeError:
            return default

    def replace(self, **changes: Any) -> "Node":
        fields = dict(self.fields)
        positional = list(self.positional)
        names = CONSTRUCTORS.get(self.kind, ())
        for key, value in changes.items():
            if key in fields:
                fields[key] = value
            elif key in names:
                positional[names.index(key)] = value
            else:
                raise IRError(f"{self.kind} has no field {key!r}")
        return Node(self.kind, tuple(positional), fields)

    def __eq__(self, other: object) -> bool:
        return (isinstance(other, Node) and self.kind == other.kind
                and self.positional == other.positional and self.fields == other.fields)

    def __hash__(self) -> int:
        return hash(render(self))

    def __repr__(self) -> str:
        return render(self)


def render(value: Any) -> str:
    """Serialise a value exactly as the Kernel-IR format writes it."""
    if isinstance(value, Node):
        parts = [render(v) for v in value.positional]
        parts += [f"{k}={render(v)}" for k, v in value.fields.items()]
        return f"{value.kind}({', '.join(parts)})"
    if isinstance(value, tuple):
        if len(value) == 1:
            return f"({render(value[0])},)"
        return "(" + ", ".join(render(v) for v in value) + ")"
    if isinstance(value, list):
        return "[" + ", ".join(render(v) for v in value) + "]"
    return repr(value)


def _convert(node: ast.AST, depth: int = 0) -> Any:
    if depth > 400:
        raise IRError("IR expression nests too deeply")
    if isinstance(node, ast.Constant):
        if isinstance(node.value, (str, int, float, bool)) or node.value is None:
            return node.value
        raise IRError(f"unsupported constant {node.value!r}")
    if isinstance(node, ast.Name) and node.id in ("inf", "nan"):
        # ``repr`` of a non-finite float (e.g. a max-fold identity of -inf).
        return float(node.id)
    if isinstance(node, ast.UnaryOp) and isinstance(node.op, (ast.USub, ast.UAdd)):
        inner = _convert(node.operand, depth + 1)
        if isinstance(inner, bool) or not isinstance(inner, (int, float)):
            raise IRError("unary sign on a non-number")
        return -inner if isinstance(node.op, ast.USub) else +inner
    if isinstance(node, ast.Tuple):
        return tuple(_convert(e, depth + 1) for e in node.elts)
    if isinstance(node, ast.List):
        return [_convert(e, depth + 1) for e in node.elts]
    if isinstance(node, ast.Call):
        if not isinstance(node.func, ast.Name) or node.func.id not in CONSTRUCTORS:
            raise IRError(f"unknown constructor {ast.dump(node.func)[:80]}")
        kind = node.func.id
        positional = tuple(_convert(a, depth + 1) for a in node.args)
        if len(positional) > len(CONSTRUCTORS[kind]):
            raise IRError(f"{kind} takes no positional argument beyond {CONSTRUCTORS[kind]}")
        fields = {}
        for kw in node.keywords:
            if kw.arg is None or kw.arg in fields:
                raise IRError(f"{kind}: bad keyword")
            fields[kw.arg] = _convert(kw.value, depth + 1)
        return Node(kind, positional, fields)
    raise IRError(f"unsupported IR syntax {type(node).__name__}")


def parse(text: str) -> Node:
    """Parse one serialised statement into a :class:`Node` tree."""
    if not isinstance(text, str) or len(text) > MAX_SOURCE:
        raise IRError("statement text must be a string of bounded size")
    try:
        tree = ast.parse(text, mode="eval")
    except SyntaxError as exc:
        raise IRError(f"statement is not valid Kernel-IR: {exc.msg}") from exc
    value = _convert(tree.body)
    if not isinstance(value, Node) or value.kind not in STATEMENTS:
        raise IRError("a kernel body entry must be one statement")
    return value


class GraphNode:
    """One graph node: an ``InputOp``, ``ConstantOp`` or ``KernelOp``."""

    def __init__(self, name: str, op: str, fields: dict, inputs: list, outputs: list, raw: dict):
        self.name, self.op, self.fields = name, op, fields
        self.inputs, self.outputs, self._raw = inputs, outputs, raw
        self.body: tuple[Node, ...] = ()
        if op == "KernelOp":
            body = fields.get("body")
            if not isinstance(body, list):
                raise IRError(f"KernelOp {name!r} has no body list")
            self.body = tuple(parse(s) for s in body)

    @property
    def entry(self) -> str | None:
        return self.fields.get("name")

    def buffer_names(self) -> list[str]:
        return [o["name"] for o in self.outputs]

    def to_dict(self) -> dict:
        fields = dict(self.fields)
        if self.op == "KernelOp":
            fields["body"] = [render(s) for s in self.body]
        return {**self._raw, "op_fields": fields}


class Graph:
    """A loaded Kernel-IR graph (the replacement for emmy's ``Graph``)."""

    def __init__(self, inputs: list, outputs: list, nodes: dict[str, GraphNode], raw: dict):
        self.inputs, self.outputs, self.nodes, self._raw = inputs, outputs, nodes, raw

    @classmethod
    def from_dict(cls, data: dict) -> "Graph":
        if not isinstance(data, dict) or not isinstance(data.get("nodes"), dict):
            raise IRError("graph JSON needs a 'nodes' object")
        nodes = {}
        for name, raw in data["nodes"].items():
            if not isinstance(raw, dict) or raw.get("op") not in ("InputOp", "ConstantOp", "KernelOp"):
                raise IRError(f"node {name!r} has an unsupported op")
            outputs = raw.get("outputs", [])
            for out in outputs:
                if not isinstance(out, dict) or not isinstance(out.get("name"), str):
                    raise IRError(f"node {name!r} has a malformed output")
            nodes[name] = GraphNode(name, raw["op"], dict(raw.get("op_fields", {})),
                                    list(raw.get("inputs", [])), list(outputs), raw)
        return cls(list(data.get("inputs", [])), list(data.get("outputs", [])), nodes, data)

    @classmethod
    def load(cls, path: str | Path) -> "Graph":
        return cls.from_dict(json.loads(Path(path).read_text()))

    def to_dict(self) -> dict:
        return {**self._raw, "nodes": {k: n.to_dict() for k, n in self.nodes.items()}}

    def kernels(self) -> list[GraphNode]:
        return [n for n in self.nodes.values() if n.op == "KernelOp"]

    def tensor(self, name: str) -> dict | None:
        """The declared ``{name, shape, dtype}`` of a graph tensor."""
        for node in self.nodes.values():
            for out in node.outputs:
                if out["name"] == name:
                    return out
        return None


# --- traversal helpers -------------------------------------------------------

BODY_FIELDS = ("body", "else_body", "combine_states")


def children(stmt: Node) -> Iterator[tuple[str, tuple]]:
    for field in BODY_FIELDS:
        value = stmt.fields.get(field)
        if isinstance(value, tuple):
            yield field, value
    if stmt.kind == "Select":
        for branch in stmt.fields.get("branches", ()) or ():
            if isinstance(branch, Node):
                yield "branch", (branch,)


def walk(statements: Iterable[Node]) -> Iterator[Node]:
    """Pre-order walk over every statement, including nested bodies."""
    for stmt in statements:
        if not isinstance(stmt, Node):
            continue
        yield stmt
        for _, body in children(stmt):
            yield from walk(body)


def static_int(value: Any) -> int:
    """A static integer from ``Dim(n)``, ``Literal(n)`` or an int."""
    if isinstance(value, bool):
        raise IRError("boolean is not a static integer")
    if isinstance(value, int):
        return value
    if isinstance(value, Node) and value.kind == "Dim":
        return static_int(value.value)
    if isinstance(value, Node) and value.kind == "Literal" and isinstance(value.value, int):
        return value.value
    raise IRError(f"expected a static integer, got {value!r}")
