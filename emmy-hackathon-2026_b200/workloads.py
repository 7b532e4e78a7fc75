"""Seeded synthetic inputs for the five benchmark configurations.

The reference measures on small published problems and seeded scaled cases
(tests/performance/generators/suite.py:284-310 draws inputs with
``numpy.random.default_rng(seed)``); the configurations benchmarked here are
larger and are described in prose, so their inputs are drawn the same way
with fixed seeds and the stated distributions:

* add        -- a, b ~ U[-1, 1], n = 2^24                       (seeds 1001, 1002)
* softmax    -- x ~ N(0, var 16), 4096 x 8192, 1 % of the entries
                (seeded choice) set to -100                      (seeds 2001, 2002)
* gemm       -- A, B ~ U[-1, 1], 4096^3, row-major              (seeds 1001, 1002)
* ragged     -- A 4097 x 777, B^T 1000 x 777 ~ N(0, 1),
                bias[1000] ~ U[-0.5, 0.5]                        (seeds 1001, 1002, 4001)
* attention  -- Q, K, V ~ N(0, 1), [64 = 4 batches x 16 heads, 2048, 128]
                                                                 (seeds 3001, 3002, 3003)
"""
from __future__ import annotations

from pathlib import Path

import numpy as np

F32 = np.float32

CONFIGS = {
    "add": {"n": 1 << 24},
    "softmax": {"rows": 4096, "cols": 8192},
    "gemm": {"m": 4096, "n": 4096, "k": 4096},
    "ragged": {"m": 4097, "n": 1000, "k": 777},
    "attention": {"batch": 4, "heads": 16, "seq": 2048, "head_dim": 128},
}


def rng(seed: int) -> np.random.Generator:
    return np.random.default_rng(seed)


def add_inputs(n: int = 1 << 24) -> tuple[np.ndarray, np.ndarray]:
    return (rng(1001).uniform(-1, 1, n).astype(F32), rng(1002).uniform(-1, 1, n).astype(F32))


def softmax_input(rows: int = 4096, cols: int = 8192) -> np.ndarray:
    x = rng(2001).normal(0.0, 4.0, (rows, cols)).astype(F32)
    count = max(1, (rows * cols) // 100)
    picked = rng(2002).choice(rows * cols, size=count, replace=False)
    x.reshape(-1)[picked] = F32(-100.0)
    return x


def gemm_inputs(m: int = 4096, n: int = 4096, k: int = 4096) -> tuple[np.ndarray, np.ndarray]:
    return (rng(1001).uniform(-1, 1, (m, k)).astype(F32), rng(1002).uniform(-1, 1, (k, n)).astype(F32))


def ragged_inputs(m: int = 4097, n: int = 1000, k: int = 777) -> tuple[np.ndarray, np.ndarray, np.ndarray]:
    return (rng(1001).standard_normal((m, k)).astype(F32),
            rng(1002).standard_normal((n, k)).astype(F32),
            rng(4001).uniform(-0.5, 0.5, n).astype(F32))


def attention_inputs(bh: int = 64, seq: int = 2048, d: int = 128) -> tuple[np.ndarray, np.ndarray, np.ndarray]:
    return tuple(rng(s).standard_normal((bh, seq, d)).astype(F32) for s in (3001, 3002, 3003))


# Algorithmic work per run (bytes or flop), the roofline numerators.
def add_bytes(n: int = 1 << 24) -> int:
    return 3 * 4 * n


def softmax_bytes(rows: int = 4096, cols: int = 8192) -> int:
    return 2 * 4 * rows * cols


def gemm_flop(m: int, n: int, k: int) -> int:
    return 2 * m * n * k


def attention_flop(bh: int, seq: int, d: int) -> int:
    return 4 * bh * seq * seq * d


# --------------------------------------------------------------------------- scaled Kernel IR
# The reference scales its published IRs to benchmark sizes by rewriting only
# the shape-bearing fields -- tensor shapes, Tile / Loop axis extents, window
# parents, the launch grid and the seeded metadata -- never the schedule
# (tests/performance/generators/suite.py:313-393 generate_case, with
# _rename_and_rescale :103-147 and the per-family extents and grids
# :349-370).  scaled_case does the same on this package's typed IR (ir.py)
# so that BASELINE-sized kernels can go through the front end
# (frontend.compile_path) and b2k_launch.  Families:
#
#   add        template p01_vector_add   shape (n,)        a0 = n / vector width, grid = a0 / block
#   softmax    template f02_row_softmax  shape (rows, cols) a0 = rows, a1..a3 = cols, grid = rows
#   gemm       template m01_matmul_512   shape (m, n, k)   a0_b = m / 32, a1_b = n / 64, _ks = k,
#                                                          windows a0 = m, a1 = n, grid = m/32 * n/64;
#                                                          the reference scales only M and N of this
#                                                          schedule (its perf cases keep K = 512), whose
#                                                          cp.async prefetch guard holds K as literals
#                                                          (_ks + 128 < K ? _ks + 128 : K - 64): those two
#                                                          literals are rewritten for the new K as well
#   attention  template a01_attention    shape (seq, width) a0_b = seq / 32, a5_b = width / 32, a1 = seq,
#                                                          a2 = width (the reference keeps width 64 and
#                                                          does not list a2; here the head dim changes
#                                                          too), div_c1 = sqrt(width)
#   matmul     any template              explicit extents, windows, grid and tensor shapes
def _rescale_stmt(node, extents: dict, windows: dict):
    from .ir import Node, children

    def dim(n):
        return Node("Dim", (int(n),), {})

    def axis(a):
        fields = dict(a.fields)
        if a.name in extents:
            fields["extent"] = dim(extents[a.name])
        w = fields.get("window")
        if isinstance(w, Node) and isinstance(w.get("parent"), Node) and w.parent.name in windows:
            parent = w.parent.replace(extent=dim(windows[w.parent.name]))
            fields["window"] = w.replace(parent=parent)
        return Node(a.kind, a.positional, fields)

    if node.kind == "Tile":
        node = node.replace(axes=tuple(axis(a) for a in node.axes))
    elif node.kind in ("Loop", "StridedLoop"):
        node = node.replace(axis=axis(node.axis))
    changes = {field: tuple(_rescale_stmt(s, extents, windows) if isinstance(s, Node) else s for s in body)
               for field, body in children(node) if field in ("body", "else_body")}
    return node.replace(**changes) if changes else node


def _rewrite_guard_literals(value, axis: str, literals: dict):
    """Replace the integer literals in `literals` inside every TernaryExpr whose
    condition reads `axis` (a loop-bound guard), anywhere under `value`."""
    from .ir import Node

    def reads(e):
        if isinstance(e, Node):
            if e.kind == "Var" and e.name == axis:
                return True
            return any(reads(v) for v in e.positional) or any(reads(v) for v in e.fields.values())
        if isinstance(e, (tuple, list)):
            return any(reads(v) for v in e)
        return False

    def swap(e):
        if isinstance(e, Node):
            if e.kind == "Literal" and isinstance(e.value, int) and not isinstance(e.value, bool) \
                    and e.value in literals:
                return e.replace(value=literals[e.value])
            return Node(e.kind, tuple(swap(v) for v in e.positional), {k: swap(v) for k, v in e.fields.items()})
        if isinstance(e, tuple):
            return tuple(swap(v) for v in e)
        if isinstance(e, list):
            return [swap(v) for v in e]
        return e

    def visit(e):
        if isinstance(e, Node):
            if e.kind == "TernaryExpr" and reads(e.cond):
                return swap(e)
            return Node(e.kind, tuple(visit(v) for v in e.positional), {k: visit(v) for k, v in e.fields.items()})
        if isinstance(e, tuple):
            return tuple(visit(v) for v in e)
        if isinstance(e, list):
            return [visit(v) for v in e]
        return e
    return visit(value)


def rescale_graph(graph: dict, shapes: dict, extents: dict, windows: dict | None = None,
                  guards: tuple | None = None) -> dict:
    """A copy of an IR graph (JSON dict) with tensor shapes, axis extents and
    window parents rewritten; statements are otherwise unchanged."""
    import copy

    from .ir import parse, render
    graph = copy.deepcopy(graph)
    for node in graph["nodes"].values():
        for out in node.get("outputs", []):
            if out["name"] in shapes:
                out["shape"] = [int(s) for s in shapes[out["name"]]]
        if node.get("op") == "KernelOp":
            body = node["op_fields"]["body"]
            stmts = [_rescale_stmt(parse(s), extents, windows or {}) for s in body]
            if guards:
                stmts = [_rewrite_guard_literals(st, guards[0], guards[1]) for st in stmts]
            node["op_fields"]["body"] = [render(st) for st in stmts]
    return graph


def scaled_case(template, out, family: str, shape, seed: int = 20260101) -> Path:
    """Write ``out/meta.json`` and ``out/<entry>.ir.json``: the published IR in
    ``template`` rescaled to ``shape`` for ``family`` (see the table above).
    Inputs without fixed data get seeds ``seed``, ``seed + 1``, ... in argument
    order, as the reference's scaled metadata does (suite.py:262-281)."""
    import json
    import math
    template, out = Path(template), Path(out)
    meta = json.loads((template / "meta.json").read_text())
    ir_path = next(template.glob("*.ir.json"))
    graph = json.loads(ir_path.read_text())
    kernel = meta["kernels"][0]
    args = {a["name"]: a for a in kernel["args"]}
    windows: dict = {}
    guards = None
    if family == "add":
        (n,) = shape
        shapes = {name: (n,) for name in args}
        old_n = args[kernel["arg_order"][0]]["shape"][0]
        tile = _tile_extent(graph, "a0")
        width = old_n // tile
        extents = {"a0": math.ceil(n / width)}
        grid = math.ceil(extents["a0"] / math.prod(kernel["block"]))
    elif family == "softmax":
        rows, cols = shape
        shapes = {name: (rows, cols) for name in args}
        extents = {"a0": rows, "a1": cols, "a2": cols, "a3": cols}
        grid = rows
    elif family == "gemm":
        m, n, k = shape
        if m % 32 or n % 64 or k % 64:
            raise ValueError("the m01 schedule tiles M by 32, N by 64 and K by 64")
        shapes = {"x0": (m, k), "x1": (k, n), "matmul": (m, n)}
        extents = {"a0_b": m // 32, "a1_b": n // 64, "_ks": k}
        windows = {"a0": m, "a1": n}
        grid = (m // 32) * (n // 64)
        k_old = args["x0"]["shape"][1]
        guards = ("_ks", {k_old: k, k_old - 64: k - 64})
    elif family == "attention":
        seq, width = shape
        shapes = {"q": (seq, width), "kt": (width, seq), "v": (seq, width), "matmul_1": (seq, width)}
        extents = {"a0_b": math.ceil(seq / 32), "a5_b": math.ceil(width / 32), "a1": seq, "a2": width}
        grid = math.ceil(seq / 32) * math.ceil(width / 32)
        args["div_c1"]["data"] = [math.sqrt(width)]
    else:
        raise ValueError(f"unknown family {family!r}")
    graph = rescale_graph(graph, shapes, extents, windows, guards)
    index = 0
    for name in kernel["arg_order"]:
        arg = args[name]
        if name in shapes:
            arg["shape"] = [int(s) for s in shapes[name]]
        if not arg.get("output") and "data" not in arg:
            arg["seed"] = seed + index
            index += 1
    kernel["grid"] = [int(grid), 1, 1]
    meta["id"] = f"{meta.get('id', family)}_scaled_" + "x".join(str(s) for s in shape)
    out.mkdir(parents=True, exist_ok=True)
    (out / "meta.json").write_text(json.dumps(meta, indent=1))
    dest = out / f"{kernel['entry']}.ir.json"
    dest.write_text(json.dumps(graph))
    return dest


def _tile_extent(graph: dict, axis: str) -> int:
    from .ir import parse, static_int, walk
    for node in graph["nodes"].values():
        if node.get("op") == "KernelOp":
            for s in walk(parse(b) for b in node["op_fields"]["body"]):
                if s.kind == "Tile":
                    for a in s.axes:
                        if a.name == axis:
                            return static_int(a.extent)
    raise ValueError(f"no Tile axis {axis!r}")
