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


def _is_int(v) -> bool:
    return isinstance(v, (int, np.integer)) or (isinstance(v, np.ndarray) and v.dtype.kind in "iu")


def _trunc_div(a, b):
    a = np.asarray(a, dtype=np.int64)
    b = np.asarray(b, dtype=np.int64)
    q = np.abs(a) // np.where(b == 0, 1, np.abs(b))
    return np.where((a < 0) ^ (b < 0), -q, q)


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
