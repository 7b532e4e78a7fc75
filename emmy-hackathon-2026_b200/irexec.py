"""Lockstep execution of Kernel-IR for a few CTAs, used by the recogniser.

The recogniser (``frontend.classify``) decides which B200 kernel computes a
given IR kernel.  Besides structural checks it runs the IR itself on seeded
random inputs for a sample of CTAs and compares what those CTAs write with
the candidate kernel family's mathematics.  This module is that executor: it
follows the statement semantics of the reference's lowering (Tile decode
``compile.py:8473-8585``; loops, Accum seeding and carried state
``compile.py:8404-9270``; cp.async transport ``compile.py:9041-9127``;
WarpShuffle butterflies ``compile.py:8958-9035``; TreeHalve trees
``compile.py:9175-9268``) with every thread of the sampled CTAs held as one
lane of NumPy arrays, so barriers are implicit (lockstep).  It never produces
a kernel's output for the caller: recognised kernels always run on the GPU.
"""
from __future__ import annotations

import math
from dataclasses import dataclass, field

import numpy as np

from .ir import IRError, Node, static_int


class ExecError(ValueError):
    """The IR uses a construct this executor does not model, or misbehaves."""


def _identity(op: str) -> float:
    return {"add": 0.0, "multiply": 1.0, "maximum": -math.inf, "minimum": math.inf}.get(op, 0.0)


def _elementwise(op: str, args: list):
    a = args[0]
    b = args[1] if len(args) > 1 else None
    with np.errstate(all="ignore"):
        if op in ("add", "plus"):
            return a + b
        if op == "subtract":
            return a - b
        if op == "multiply":
            return a * b
        if op in ("divide", "true_divide"):
            return np.divide(a, b)
        if op in ("maximum", "max"):
            return np.maximum(a, b)
        if op in ("minimum", "min"):
            return np.minimum(a, b)
        if op in ("negative", "negate"):
            return -a
        if op == "reciprocal":
            return np.divide(1.0, a)
        if op == "sqrt":
            return np.sqrt(a)
        if op in ("rsqrt", "reciprocal_sqrt"):
            return np.divide(1.0, np.sqrt(a))
        if op in ("exp", "exp_fast"):
            return np.exp(a)
        if op in ("identity", "copy"):
            return a
        if op == "relu":
            return np.maximum(a, 0.0)
        if op == "abs":
            return np.abs(a)
        if op == "greater":
            return (a > b).astype(np.float64)
        if op == "greater_equal":
            return (a >= b).astype(np.float64)
        if op == "less":
            return (a < b).astype(np.float64)
        if op == "less_equal":
            return (a <= b).astype(np.float64)
        if op == "where":
            return np.where(a != 0, b, args[2])
        if op == "log":
            return np.log(a)
    raise ExecError(f"elementwise op {op!r} is outside the hot path")


@dataclass
class Launch:
    grid: int
    block: int
    ctas: np.ndarray            # sampled CTA indices
    buffers: dict               # name -> float64 array (global)
    shapes: dict                # name -> shape
    writes: dict = field(default_factory=dict)   # name -> int count array (global writes)
    max_statements: int = 5_000_000


class CTAExecutor:
    """Executes a kernel body for the sampled CTAs of a launch, in lockstep."""

    def __init__(self, launch: Launch):
        self.L = launch
        nct = len(launch.ctas)
        self.nlanes = nct * launch.block
        self.tid = np.tile(np.arange(launch.block, dtype=np.int64), nct)
        self.bid = np.repeat(launch.ctas.astype(np.int64), launch.block)
        self.cta_slot = np.repeat(np.arange(nct, dtype=np.int64), launch.block)
        self.gid = self.bid * launch.block + self.tid
        self.smem: dict = {}
        self.smem_shapes: dict = {}
        self.budget = launch.max_statements

    # --- expressions -----------------------------------------------------------
    def expr(self, e, env):
        if isinstance(e, bool):
            return e
        if isinstance(e, (int, float)):
            return e
        if not isinstance(e, Node):
            raise ExecError(f"unexpected expression {e!r}")
        k = e.kind
        if k == "Var":
            name = e.name
            if name in env:
                return env[name]
            if name == "tid":
                return self.tid
            if name == "lane":
                return self.tid % 32
            if name == "warp":
                return self.tid // 32
            raise ExecError(f"unbound variable {name!r}")
        if k == "Literal":
            return e.value
        if k == "Dim":
            return static_int(e)
        if k == "TernaryExpr":
            c = self.expr(e.cond, env)
            return np.where(c, self.expr(e.if_true, env), self.expr(e.if_false, env))
        if k == "BinaryExpr":
            a, b = self.expr(e.left, env), self.expr(e.right, env)
            op = e.op
            if op == "+":
                return a + b
            if op == "-":
                return a - b
            if op == "*":
                return a * b
            if op == "/":
                if _is_int(a) and _is_int(b):
                    return _trunc_div(a, b)
                with np.errstate(all="ignore"):
                    return np.divide(a, b)
            if op == "//":
                return np.floor_divide(a, b)
            if op == "%":
                return np.mod(a, b)
            if op == "<":
                return a < b
            if op == "<=":
                return a <= b
            if op == ">":
                return a > b
            if op == ">=":
                return a >= b
            if op == "==":
                return a == b
            if op == "!=":
                return a != b
            if op in ("&&", "and"):
                return np.logical_and(a, b)
            if op in ("||", "or"):
                return np.logical_or(a, b)
            raise ExecError(f"operator {op!r}")
        if k == "Builtin":
            name = e.name
            if name == "thread_idx.x":
                return self.tid
            if name == "block_idx.x":
                return self.bid
            if name == "block_dim.x":
                return self.L.block
            if name == "grid_dim.x":
                return self.L.grid
            if name.endswith((".y", ".z")):
                return 0 if "idx" in name else 1
            raise ExecError(f"builtin {name!r}")
        if k == "FuncCallExpr":
            args = [self.expr(a, env) for a in e.args]
            if e.name == "minimum":
                return np.minimum(args[0], args[1])
            if e.name == "maximum":
                return np.maximum(args[0], args[1])
            if e.name == "abs":
                return np.abs(args[0])
            raise ExecError(f"function {e.name!r}")
        if k == "CastExpr":
            v = self.expr(e.expr, env)
            if e.dtype in ("int", "i32", "i64"):
                return np.trunc(np.asarray(v, dtype=np.float64)).astype(np.int64)
            return np.asarray(v, dtype=np.float64)
        raise ExecError(f"expression kind {k!r} is outside the hot path")

    # --- memory -----------------------------------------------------------------
    def _flat(self, shape, index, env):
        if len(index) == 0 and int(np.prod(shape)) == 1:
            return np.zeros(self.nlanes, dtype=np.int64)
        if len(index) != len(shape):
            raise ExecError("index rank differs from buffer rank")
        flat = 0
        for dim, e in zip(shape, index):
            flat = flat * int(dim) + np.asarray(self.expr(e, env), dtype=np.int64)
        return np.broadcast_to(np.asarray(flat, dtype=np.int64), (self.nlanes,))

    def _buffer(self, name):
        if name in self.smem:
            return self.smem[name], self.smem_shapes[name], True
        if name in self.L.buffers:
            return self.L.buffers[name], self.L.shapes[name], False
        raise ExecError(f"unknown buffer {name!r}")

    def load(self, name, flat, mask):
        buf, shape, shared = self._buffer(name)
        size = int(np.prod(shape)) if len(shape) else 1
        f = np.where(mask, flat, 0)
        if np.any(mask & ((flat < 0) | (flat >= size))):
            raise ExecError(f"out-of-bounds read of {name!r}")
        if shared:
            return buf[self.cta_slot, f]
        return buf.reshape(-1)[f]

    def store(self, name, flat, values, mask, atomic=False):
        buf, shape, shared = self._buffer(name)
        size = int(np.prod(shape)) if len(shape) else 1
        if np.any(mask & ((flat < 0) | (flat >= size))):
            raise ExecError(f"out-of-bounds write of {name!r}")
        idx = np.nonzero(mask)[0]
        if idx.size == 0:
            return
        vals = np.broadcast_to(np.asarray(values, dtype=np.float64), (self.nlanes,))[idx]
        f = flat[idx]
        if shared:
            if atomic:
                np.add.at(buf, (self.cta_slot[idx], f), vals)
            else:
                buf[self.cta_slot[idx], f] = vals
            return
        flat_buf = buf.reshape(-1)
        if atomic:
            np.add.at(flat_buf, f, vals)
        else:
            flat_buf[f] = vals
        counts = self.L.writes.setdefault(name, np.zeros(size, dtype=np.int64))
        np.add.at(counts, f, 1)

    # --- statements ---------------------------------------------------------------
    def run(self, body, env, mask):
        for stmt in body:
            self.stmt(stmt, env, mask)

    def _assign(self, env, name, value, mask):
        value = np.broadcast_to(np.asarray(value), (self.nlanes,))
        old = env.get(name)
        if old is None:
            env[name] = np.array(value, dtype=np.float64 if value.dtype.kind == "f" else value.dtype)
        else:
            env[name] = np.where(mask, value, old)

    def _seed(self, body, env, mask):
        for stmt in body:
            if stmt.kind == "Accum":
                self._assign(env, stmt.name, _identity(stmt.op.name), mask)
            elif stmt.kind == "Cond":
                self._seed(stmt.body, env, mask)
                self._seed(stmt.else_body, env, mask)

    def stmt(self, s: Node, env, mask):
        self.budget -= 1
        if self.budget < 0:
            raise ExecError("execution budget exhausted")
        k = s.kind
        if k == "Tile":
            if s.get("aux_threads", 0):
                raise ExecError("auxiliary Tile threads")
            extents = [static_int(a.extent) for a in s.axes]
            n = math.prod(extents)
            active = mask & (self.gid < n)
            for i, axis in enumerate(s.axes):
                stride = math.prod(extents[i + 1:])
                v = self.gid // stride
                if i:
                    v = v % extents[i]
                env[axis.name] = v
            self.run(s.body, env, active)
        elif k == "Loop":
            if s.get("seed"):
                self._seed(s.body, env, mask)
            if _fold_loop(s):
                self._run_fold_loop(s, env, mask)
                return
            for v in range(static_int(s.axis.extent)):
                env[s.axis.name] = np.full(self.nlanes, v, dtype=np.int64)
                self.run(s.body, env, mask)
        elif k == "StridedLoop":
            if s.get("seed"):
                self._seed(s.body, env, mask)
            start = np.broadcast_to(np.asarray(self.expr(s.start, env), dtype=np.int64), (self.nlanes,))
            step = int(np.max(self.expr(s.step, env)))
            end = static_int(s.axis.extent) if s.get("end") is None else self.expr(s.end, env)
            if step <= 0:
                raise ExecError("non-positive loop step")
            it = 0
            while True:
                value = start + it * step
                m = mask & (value < end)
                if not m.any():
                    break
                env[s.axis.name] = value
                self.run(s.body, env, m)
                it += 1
        elif k == "Load":
            flat = self._flat(self._buffer(s.input)[1], s.index, env)
            for off, name in enumerate(s.names):
                self._assign(env, name, self.load(s.input, flat + off, mask), mask)
        elif k == "Write":
            flat = self._flat(self._buffer(s.output)[1], s.index, env)
            for off, name in enumerate(s.values):
                self.store(s.output, flat + off, env[name], mask, atomic=bool(s.get("atomic")))
        elif k == "Assign":
            self._assign(env, s.name, _elementwise(s.op.name, [env[a] for a in s.args]), mask)
        elif k == "Accum":
            base = s.base or s.name
            if base not in env:
                raise ExecError(f"accumulator {base!r} read before it is seeded")
            self._assign(env, s.name, _elementwise(s.op.name, [env[base], env[s.value]]), mask)
        elif k == "Init":
            self._assign(env, s.name, self.expr(s.identity, env), mask)
        elif k == "Let":
            self._assign(env, s.name, self.expr(s.value, env), mask)
        elif k == "Cond":
            c = np.broadcast_to(np.asarray(self.expr(s.cond, env), dtype=bool), (self.nlanes,))
            self.run(s.body, env, mask & c)
            self.run(s.else_body, env, mask & ~c)
        elif k == "Smem":
            shape = tuple(static_int(e) for e in s.extents)
            self.smem[s.name] = np.full((len(self.L.ctas), int(np.prod(shape))), np.nan)
            self.smem_shapes[s.name] = shape
        elif k in ("Sync", "CpAsyncCommit", "CpAsyncWait"):
            pass
        elif k == "CpAsyncCopy":
            if s.get("swizzle") not in (None, "NONE"):
                raise ExecError("swizzled async copy")
            dst_index = s.smem_index
            if s.get("lane_index") is not None:
                dst_index = tuple(Node("BinaryExpr", (), {"op": "+", "left": a, "right": b})
                                  for a, b in zip(s.smem_index, s.lane_index))
            width = int(s.nbytes) // 4
            src_flat = self._flat(self._buffer(s.src)[1], s.src_index, env)
            dst_flat = self._flat(self._buffer(s.smem)[1], dst_index, env)
            for j in range(width):
                self.store(s.smem, dst_flat + j, self.load(s.src, src_flat + j, mask), mask)
        elif k == "WarpShuffle":
            length = int(s.length)
            offset = length // 2
            while offset:
                partner = (self.tid // 32) * 32 + ((self.tid % 32) ^ offset) + self.cta_slot * self.L.block
                for name, other in zip(s.state, s.state_b):
                    env[other] = np.asarray(env[name])[partner]
                self.run(s.combine_states, env, mask | True)
                offset //= 2
        elif k == "TreeHalve":
            self._tree_halve(s, env)
        else:
            raise ExecError(f"statement {k!r} is outside the hot path")

    # --- fold loops, all iterations at once -----------------------------------------
    def _run_fold_loop(self, s, env, mask):
        """A Loop whose body only loads, computes and folds into accumulators
        (a dot product over K, a sum over keys): every iteration of a chunk is
        evaluated at once as a second array axis, and each accumulator takes
        its chunk's fold in iteration order -- the same mathematics as the
        serial loop, with the folds of one chunk reassociated (float64, far
        inside the certificate's tolerance).  Names the body defines keep the
        last iteration's value, as after the serial loop."""
        extent = static_int(s.axis.extent)
        if extent <= 0:
            return
        n = self.nlanes
        chunk = max(1, min(extent, 4_000_000 // max(1, n)))
        saved = (self.tid, self.bid, self.gid)
        self.tid, self.bid, self.gid = self.tid[:, None], self.bid[:, None], self.gid[:, None]
        m2 = mask[:, None]
        last: dict = {}
        try:
            for c0 in range(0, extent, chunk):
                c1 = min(extent, c0 + chunk)
                self.budget -= len(s.body)
                if self.budget < 0:
                    raise ExecError("execution budget exhausted")
                venv = _ColumnView(env, n)
                venv[s.axis.name] = np.arange(c0, c1, dtype=np.int64)[None, :]
                shape2 = (n, c1 - c0)
                for st in s.body:
                    if st.kind == "Load":
                        buf, bshape, shared = self._buffer(st.input)
                        size = int(np.prod(bshape)) if len(bshape) else 1
                        if len(st.index) == 0 and size == 1:
                            flat = np.zeros(shape2, dtype=np.int64)
                        else:
                            if len(st.index) != len(bshape):
                                raise ExecError("index rank differs from buffer rank")
                            flat = 0
                            for dim, e in zip(bshape, st.index):
                                flat = flat * int(dim) + np.asarray(self.expr(e, venv), dtype=np.int64)
                            flat = np.broadcast_to(np.asarray(flat, dtype=np.int64), shape2)
                        for off, name in enumerate(st.names):
                            f = flat + off
                            if np.any(m2 & ((f < 0) | (f >= size))):
                                raise ExecError(f"out-of-bounds read of {st.input!r}")
                            f = np.where(m2, f, 0)
                            venv[name] = buf[self.cta_slot[:, None], f] if shared else buf.reshape(-1)[f]
                            last[name] = True
                    elif st.kind == "Assign":
                        venv[st.name] = _elementwise(st.op.name, [venv[a] for a in st.args])
                        last[st.name] = True
                    elif st.kind == "Let":
                        venv[st.name] = self.expr(st.value, venv)
                        last[st.name] = True
                    else:  # Accum: fold this chunk's values in order into the accumulator
                        base = st.base or st.name
                        if base not in env:
                            raise ExecError(f"accumulator {base!r} read before it is seeded")
                        vals = np.broadcast_to(np.asarray(venv[st.value], dtype=np.float64), shape2)
                        op = st.op.name
                        with np.errstate(all="ignore"):
                            part = {"add": np.sum, "multiply": np.prod, "maximum": np.max,
                                    "minimum": np.min}[op](vals, axis=1)
                        self._assign(env, st.name, _elementwise(op, [np.asarray(env[base]), part]), mask)
                        venv[st.name] = np.asarray(env[st.name])[:, None]
                for name in last:
                    value = np.broadcast_to(np.asarray(venv[name]), shape2)[:, -1]
                    self._assign(env, name, value, mask)
            env[s.axis.name] = np.full(n, extent - 1, dtype=np.int64)
        finally:
            self.tid, self.bid, self.gid = saved

    def _tree_halve(self, s, env):
        length = int(s.length)
        nct = len(self.L.ctas)
        bufs = [self.smem[b] for b in s.bufs]
        stride = length // 2
        while stride:
            sub = {}
            for buf, name, other in zip(bufs, s.state, s.state_b):
                sub[name] = buf[:, :stride].reshape(-1).copy()
                sub[other] = buf[:, stride:2 * stride].reshape(-1).copy()
            tmp = _SubExecutor(nct * stride)
            tmp.run(s.combine_states, sub)
            for buf, name in zip(bufs, s.state):
                buf[:, :stride] = np.asarray(sub[name]).reshape(nct, stride)
            stride //= 2
        for buf, name in zip(bufs, s.state):
            env[name] = buf[self.cta_slot, 0]


class _SubExecutor:
    """Runs pure combine programs (Assign only) on arrays of any length."""

    def __init__(self, n):
        self.n = n

    def run(self, body, env):
        for s in body:
            if s.kind != "Assign":
                raise ExecError("combine program with a non-Assign statement")
            env[s.name] = _elementwise(s.op.name, [env[a] for a in s.args])


class _ColumnView(dict):
    """The environment seen by a fold loop's iterations: names the body sets
    live here; anything else is read from the enclosing environment, a
    per-lane value turned into a column so it broadcasts against the
    iteration axis."""

    def __init__(self, base: dict, lanes: int):
        super().__init__()
        self.base, self.lanes = base, lanes

    def __missing__(self, key):
        value = self.base[key]
        if isinstance(value, np.ndarray) and value.shape == (self.lanes,):
            value = value[:, None]
        self[key] = value
        return value

    def __contains__(self, key) -> bool:
        return dict.__contains__(self, key) or key in self.base


_FOLD_OPS = frozenset({"add", "multiply", "maximum", "minimum"})


def expr_vars(e) -> set:
    """Variable names an index / value expression reads."""
    found: set = set()

    def visit(v):
        if isinstance(v, Node):
            if v.kind == "Var":
                found.add(v.name)
            for x in v.positional:
                visit(x)
            for x in v.fields.values():
                visit(x)
        elif isinstance(v, (tuple, list)):
            for x in v:
                visit(x)
    visit(e)
    return found


def _fold_loop(s: Node) -> bool:
    """Whether a Loop body is a pure fold: Loads, Lets and Assigns that feed
    Accums of add / multiply / maximum / minimum into accumulators that no
    other statement of the body reads (a dot product, a sum over keys)."""
    accs, local = set(), set()
    for st in s.body:
        if not isinstance(st, Node):
            return False
        if st.kind == "Load":
            local.update(st.names)
        elif st.kind in ("Assign", "Let"):
            local.add(st.name)
        elif st.kind == "Accum":
            if st.op.name not in _FOLD_OPS or st.get("base") not in (None, st.name):
                return False
            accs.add(st.name)
        else:
            return False
    if accs & local or not accs:
        return False
    for st in s.body:
        if st.kind == "Assign":
            used = set(st.args)
        elif st.kind == "Accum":
            used = {st.value}
        elif st.kind == "Load":
            used = expr_vars(st.index)
        else:
            used = expr_vars(st.value)
        if used & accs:
            return False
    return True


def _is_int(v) -> bool:
    return isinstance(v, (int, np.integer)) or (isinstance(v, np.ndarray) and v.dtype.kind in "iu")


def _trunc_div(a, b):
    a = np.asarray(a, dtype=np.int64)
    b = np.asarray(b, dtype=np.int64)
    q = np.abs(a) // np.where(b == 0, 1, np.abs(b))
    return np.where((a < 0) ^ (b < 0), -q, q)


# --------------------------------------------------------------------------- output placement
class NotProvable(ExecError):
    """Where a kernel writes depends on data, so its coverage has no index-only proof."""


def placement_slice(body, outputs) -> set:
    """The statements that decide WHERE a kernel writes its outputs: every
    Write to an output buffer, the Tile / Loop / Cond statements around them,
    and the Let statements (and loops) defining the names their indices,
    conditions and loop bounds read, transitively.  Returns their ids.  A
    name defined by a Load, Assign, Accum, Init or warp exchange -- a value
    computed from data -- raises NotProvable."""
    parent: dict = {}
    lets: dict = {}
    axes: dict = {}
    data: set = set()
    writes = []

    def visit(stmts, par):
        for st in stmts:
            if not isinstance(st, Node):
                continue
            parent[id(st)] = par
            k = st.kind
            if k == "Let":
                lets.setdefault(st.name, []).append(st)
            elif k == "Load":
                data.update(st.names)
            elif k in ("Assign", "Accum", "Init"):
                data.add(st.name)
            elif k == "WarpShuffle":
                data.update(st.state)
                data.update(st.state_b)
            elif k == "TreeHalve":
                data.update(st.state)
            elif k in ("Loop", "StridedLoop"):
                axes.setdefault(st.axis.name, []).append(st)
            elif k == "Tile":
                for a in st.axes:
                    axes.setdefault(a.name, []).append(st)
            elif k == "Write" and st.output in outputs:
                writes.append(st)
            for sub in (st.fields.get("body"), st.fields.get("else_body")):
                if isinstance(sub, tuple):
                    visit(sub, st)
            if k == "Select":
                raise NotProvable("Select statements")

    visit(body, None)
    keep: set = set()
    needed: set = set()

    def mark(st):
        while st is not None and id(st) not in keep:
            keep.add(id(st))
            k = st.kind
            if k == "Cond":
                needed.update(expr_vars(st.cond))
            elif k == "StridedLoop":
                needed.update(expr_vars(st.start) | expr_vars(st.step) | expr_vars(st.get("end")))
            elif k == "Write":
                needed.update(expr_vars(st.index))
            elif k == "Let":
                needed.update(expr_vars(st.value))
            st = parent[id(st)]

    for w in writes:
        mark(w)
    done: set = set()
    while needed - done:
        name = next(iter(needed - done))
        done.add(name)
        if name in data:
            raise NotProvable(f"output placement depends on {name!r}, a value computed from data")
        if name in lets or name in axes:
            for st in lets.get(name, []) + axes.get(name, []):
                mark(st)
        elif name not in ("tid", "lane", "warp"):
            raise NotProvable(f"output placement reads the unbound name {name!r}")
    return keep


@dataclass
class Coverage:
    counts: dict                 # output name -> writes per element over the whole launch
    writes_per_cta: np.ndarray   # element writes each CTA performs


class _PlacementExecutor(CTAExecutor):
    """Runs only the placement slice of a kernel and counts output writes."""

    def __init__(self, launch, keep, coverage):
        super().__init__(launch)
        self.keep, self.coverage = keep, coverage

    def _buffer(self, name):
        if name in self.coverage.counts:
            return None, self.L.shapes[name], False
        return super()._buffer(name)

    def run(self, body, env, mask):
        for stmt in body:
            if isinstance(stmt, Node) and id(stmt) in self.keep:
                self.stmt(stmt, env, mask)

    def stmt(self, s: Node, env, mask):
        if s.kind != "Write":
            return super().stmt(s, env, mask)
        self.budget -= 1
        if self.budget < 0:
            raise ExecError("execution budget exhausted")
        counts = self.coverage.counts[s.output]
        flat = self._flat(self.L.shapes[s.output], s.index, env)
        idx = np.nonzero(mask)[0]
        for off in range(len(s.values)):
            f = flat[idx] + off
            if np.any((f < 0) | (f >= counts.size)):
                raise ExecError(f"out-of-bounds write of {s.output!r}")
            np.add.at(counts, f, 1)
        per_cta = np.bincount(self.cta_slot[idx], minlength=len(self.L.ctas)) * len(s.values)
        self.coverage.writes_per_cta[self.L.ctas] += per_cta


def write_coverage(body, grid: int, block: int, shapes: dict, outputs, max_lanes: int = 1 << 21,
                   max_statements: int = 2_000_000) -> Coverage:
    """Exact write counts of every output element over the WHOLE launch (every
    CTA of `grid`), from the placement slice alone -- the closed-form
    counterpart of the reference's launch enumeration (tensor_core.py:1577-1612)
    that costs a few index evaluations per lane whatever the contraction or
    row length.  CTAs run in chunks of at most `max_lanes` lanes."""
    keep = placement_slice(body, set(outputs))
    coverage = Coverage({name: np.zeros(max(1, int(np.prod(shapes[name]))), dtype=np.int64) for name in outputs},
                        np.zeros(grid, dtype=np.int64))
    per_chunk = max(1, max_lanes // max(1, block))
    budget = max_statements
    for c0 in range(0, grid, per_chunk):
        ctas = np.arange(c0, min(grid, c0 + per_chunk), dtype=np.int64)
        launch = Launch(grid=grid, block=block, ctas=ctas, buffers={}, shapes=shapes, max_statements=budget)
        ex = _PlacementExecutor(launch, keep, coverage)
        try:
            ex.run(body, {}, np.ones(ex.nlanes, dtype=bool))
        except (IRError, KeyError, IndexError, TypeError, AttributeError) as exc:
            raise ExecError(f"{type(exc).__name__}: {exc}") from exc
        budget = ex.budget
    return coverage


def execute(body, grid: int, block: int, ctas, buffers: dict, shapes: dict,
            max_statements: int = 5_000_000) -> Launch:
    """Run `body` for the given CTAs; `buffers` (float64) are updated in place."""
    launch = Launch(grid=grid, block=block, ctas=np.asarray(sorted(set(int(c) for c in ctas)), dtype=np.int64),
                    buffers=buffers, shapes=shapes, max_statements=max_statements)
    ex = CTAExecutor(launch)
    env: dict = {}
    mask = np.ones(ex.nlanes, dtype=bool)
    try:
        ex.run(body, env, mask)
    except (IRError, KeyError, IndexError, TypeError, AttributeError) as exc:
        raise ExecError(f"{type(exc).__name__}: {exc}") from exc
    return launch
