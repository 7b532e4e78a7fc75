#!/usr/bin/env python3
"""Benchmark of the B200 backend's hot path (one JSON line on rank 0).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--workload gemm|softmax|add|ragged|attention]
                    [--impl ours|reference]

A step is one pass of the hot path over one batch of synthetic input:

* ``gemm`` (default) -- the 4096^3 FP32 GEMM as 3xTF32 on tcgen05 (split
  pre-pass + tensor-core kernel), TFLOP/s of useful 2*M*N*K work;
* ``softmax`` -- row softmax of 4096 x 8192 FP32, GB/s of one read + one write;
* ``add`` -- c = a + b over 2^24 FP32, GB/s of two reads + one write;
* ``ragged`` -- relu(A B^T + bias), 4097 x 1000 x 777, TFLOP/s;
* ``attention`` -- softmax(Q K^T / sqrt(128)) V over 4 x 16 heads, S 2048,
  D 128, both contractions 3xTF32, TFLOP/s of useful 4*BH*S*S*D work.

With N > 1 (torchrun, one rank per GPU) every rank processes its own batch of
the same size (rows of A / rows of the matrix / ranges of the vector: the
partitioning the work has), so the scaling is weak and no collective is on
the data path.  ``value`` is all ranks' work over the max-over-ranks device
time.  ``e2e`` repeats the step through the public host-array API with the
inputs copied in from page-locked memory and the result copied out, every
step.  ``--impl reference`` times the reference's CPU evaluation of the same
workload (its float64 NumPy equations, restated in ``oracle/``) on the
host cores.
"""
from __future__ import annotations

import argparse
import contextlib
import importlib
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))
PKG = "emmy-hackathon-2026_b200"
METRIC = "3xTF32 FP32-GEMM TFLOP/s & pointwise/softmax GB/s at 1/2/4/8 B200 vs roofline"
L2_BYTES = 126 * 1024 * 1024


def pkg(name):
    return importlib.import_module(f"{PKG}.{name}")


def measured_peaks() -> tuple[dict, str]:
    path = ROOT / "MEASURED_PEAKS.json"
    if path.exists():
        return json.loads(path.read_text()), "measured"
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}, "fallback"


def profile_traffic(name: str) -> float | None:
    """DRAM bytes per launch of the dominant kernel from the committed ncu summary."""
    path = ROOT / "profiles" / f"{name}.md"
    if not path.exists():
        return None
    for line in path.read_text().splitlines():
        if line.startswith("dram_bytes_per_launch:"):
            try:
                return float(line.split(":", 1)[1].strip())
            except ValueError:
                return None
    return None


# --------------------------------------------------------------------------- workloads
TIMING_EVERY = 8  # steps per sampled launch of the dominant kernel


@contextlib.contextmanager
def stdout_to_stderr():
    """Point file descriptor 1 at stderr for the duration (libraries that
    write to the C-level stdout included)."""
    sys.stdout.flush()
    saved = os.dup(1)
    try:
        os.dup2(2, 1)
        yield
    finally:
        sys.stdout.flush()
        os.dup2(saved, 1)
        os.close(saved)


class Workload:
    name = ""
    unit = ""
    bound = "hbm"
    phase = ""          # library timing phase of the dominant kernel
    kernels_per_step = 2  # the dominant kernel and the operand split before it
    profile = ""

    def __init__(self, rank: int, world: int):
        self.rank, self.world = rank, world

    # work units per step (flop or bytes), the numerator of `value`
    def work(self) -> float:
        raise NotImplementedError

    def dominant_work(self) -> float:
        """Algorithmic work of one launch of the dominant kernel (roofline numerator)."""
        return self.work()

    def config(self) -> dict:
        raise NotImplementedError

    def cpu_once(self, rows: int) -> tuple[float, str]:
        raise NotImplementedError

    def cpu_extras(self) -> dict:
        """One-core figure of the same float64 sample (BLAS held to one thread),
        and, for the GEMMs, the reference's own 3xTF32 model timed on a small
        shape and extrapolated by flop."""
        extras = {}
        try:
            from threadpoolctl import threadpool_limits
            with threadpool_limits(limits=1):
                v, what = self.cpu_sample(max_seconds=2.0, rows=self.reference_rows)
            extras["single_core"] = {"value": round(v, 5), "unit": self.unit, "sample": what}
        except ImportError:
            pass
        return extras

    def cpu_sample(self, max_seconds: float = 12.0, rows: int | None = None) -> tuple[float, str]:
        """Repeat the oracle's float64 evaluation of a bounded sample for about
        `max_seconds`; returns (throughput in the metric's unit, description)."""
        rows = rows or self.default_rows
        done, work, t0 = 0, 0.0, time.perf_counter()
        while True:
            units, what = self.cpu_once(rows)
            work += units
            done += 1
            if time.perf_counter() - t0 >= max_seconds or done >= 256:
                break
        dt = time.perf_counter() - t0
        return work / dt / scale(self.unit), f"{done} x {what}"


class Gemm(Workload):
    name, unit, bound, phase = "gemm", "TFLOP/s", "tensor", "mma"
    profile = "gemm_tf32x3_4096"

    def __init__(self, rank, world, m=4096, n=4096, k=4096, ragged=False):
        super().__init__(rank, world)
        self.m, self.n, self.k, self.ragged = m, n, k, ragged

    def inputs(self):
        w = pkg("workloads")
        if self.ragged:
            return w.ragged_inputs(self.m, self.n, self.k)
        a, b = w.gemm_inputs(self.m, self.n, self.k)
        if self.rank:  # each rank owns a different slab of rows of A
            a = np.random.default_rng(1001 + 7919 * self.rank).uniform(-1, 1, a.shape).astype(np.float32)
        return a, b, None

    def work(self):
        return 2.0 * self.m * self.n * self.k

    def dominant_work(self):
        # the tensor core executes three TF32 products per useful one
        return 3.0 * self.work()

    def setup(self, ctx, torch):
        a, b, bias = self.inputs()
        self.host = (a, b, bias)
        self.da, self.db = torch.from_numpy(a).cuda(), torch.from_numpy(b).cuda()
        self.dbias = torch.from_numpy(bias).cuda() if bias is not None else None
        self.dc = torch.empty((self.m, self.n), dtype=torch.float32, device="cuda")
        self.ctx = ctx
        # the step's library call with its arguments converted once: every
        # step still runs the whole GEMM (operand split + tensor-core kernel)
        self.call = ctx.gemm_call(self.da.data_ptr(), self.db.data_ptr(), self.dc.data_ptr(), self.m, self.n,
                                  self.k, b_layout=1 if self.ragged else 0,
                                  bias=self.dbias.data_ptr() if self.dbias is not None else 0, relu=self.ragged)

    def step(self):
        self.call()

    def e2e_setup(self, session):
        a, b, bias = self.host
        self.session = session
        self.pa, self.pb = session.pinned(a.shape), session.pinned(b.shape)
        self.pa[...] = a
        self.pb[...] = b
        self.pbias = None
        if bias is not None:
            self.pbias = session.pinned(bias.shape)
            self.pbias[...] = bias
        self.pc = session.pinned((self.m, self.n))
        self.e2e_bytes = (a.nbytes + b.nbytes + (bias.nbytes if bias is not None else 0), self.pc.nbytes)

    def e2e_step(self):
        self.session.gemm_host(self.pa, self.pb, self.pc, b_layout="nk" if self.ragged else "kn",
                               bias=self.pbias, relu=self.ragged)

    def cpu_extras(self):
        extras = super().cpu_extras()
        # tf32_emitter.py:64-96's model (per-8-K atom, three FP32 accumulators),
        # restated in oracle/tf32.py, on a 256^3 slab: its cost is linear in flop.
        tf32 = importlib.import_module("oracle.tf32")
        rng = np.random.default_rng(5)
        a = rng.uniform(-1, 1, (256, 256)).astype(np.float32)
        b = rng.uniform(-1, 1, (256, 256)).astype(np.float32)
        reps, t0 = 0, time.perf_counter()
        while reps < 3 or time.perf_counter() - t0 < 1.0:
            tf32.simulate_matmul(a, b)
            reps += 1
        dt = (time.perf_counter() - t0) / reps
        extras["tf32_model"] = {"value": round(2.0 * 256 ** 3 / dt / scale(self.unit), 6), "unit": self.unit,
                                "sample": f"{reps} x oracle/tf32.simulate_matmul 256x256x256 (the reference's "
                                          "3xTF32 model, tf32_emitter.py:64-96), extrapolated by flop"}
        return extras

    def cpu_once(self, rows):
        # The oracle's float64 equations (refs.matmul / refs.matmul_bias_relu)
        # on a row slab of A.  B's float64 copy is made once and reused: a
        # full-size evaluation converts B once, so converting it again for
        # every slab would understate the reference's throughput.
        refs = importlib.import_module("oracle.refs")
        a, b, bias = self.host
        if getattr(self, "b64", None) is None:
            self.b64 = refs._f64(b).T.copy() if self.ragged else refs._f64(b)
        c = refs._f64(a[:rows]) @ self.b64
        if self.ragged:
            c = np.maximum(c + refs._f64(bias), 0.0)
        c.astype(np.float32)
        return 2.0 * rows * self.n * self.k, f"float64 NumPy matmul of a {rows}-row slab of A ({self.m}x{self.n}x{self.k})"

    default_rows = 1024
    reference_rows = 256

    def config(self):
        return {"workload": "ragged_gemm_bias_relu" if self.ragged else "gemm_3xtf32",
                "m": self.m * self.world, "m_per_gpu": self.m, "n": self.n, "k": self.k,
                "b_layout": "n_k (transposed)" if self.ragged else "k_n",
                "epilogue": "bias+relu" if self.ragged else "copy",
                "inputs": "A,B ~ N(0,1) seeded" if self.ragged else "A,B ~ U[-1,1] seeded",
                "l2": "inputs larger than L2" if (self.m * self.k + self.n * self.k) * 4 > L2_BYTES
                else "inputs smaller than L2 (split scratch 2x inputs)",
                "parallelism": f"dp{self.world} (rows of A per GPU, B replicated)"}


class Softmax(Workload):
    name, unit, bound, phase = "softmax", "GB/s", "hbm", "softmax"
    kernels_per_step = 1
    profile = "row_softmax_4096x8192"

    def __init__(self, rank, world, rows=4096, cols=8192):
        super().__init__(rank, world)
        self.rows, self.cols = rows, cols

    def work(self):
        return 2.0 * 4 * self.rows * self.cols

    def setup(self, ctx, torch):
        x = pkg("workloads").softmax_input(self.rows, self.cols)
        self.host = x
        self.ctx = ctx
        # two operand copies used alternately, as for the add: no step finds
        # the previous step's data in L2
        self.sets = []
        for _ in range(2):
            dx = torch.from_numpy(x).cuda()
            dy = torch.empty_like(dx)
            self.sets.append((dx, dy, ctx.row_softmax_call(dx.data_ptr(), dy.data_ptr(), self.rows, self.cols)))
        self.i = 0

    def step(self):
        self.sets[self.i][2]()
        self.i ^= 1

    def e2e_setup(self, session):
        self.session = session
        self.px = session.pinned(self.host.shape)
        self.px[...] = self.host
        self.py = session.pinned(self.host.shape)
        self.e2e_bytes = (self.px.nbytes, self.py.nbytes)

    def e2e_step(self):
        self.session.row_softmax_host(self.px, self.py)

    def cpu_once(self, rows):
        refs = importlib.import_module("oracle.refs")
        refs.softmax(self.host[:rows])
        return 2.0 * 4 * rows * self.cols, f"float64 NumPy stable softmax of {rows} rows x {self.cols}"

    default_rows = 512
    reference_rows = 64

    def subnormal_exp_args(self) -> int:
        """How many exp arguments x - rowmax of this input give a subnormal
        FP32 result (arguments in [-103.28, -87.34]): the range the selective
        exponential exists for."""
        if getattr(self, "_subnormal", None) is None:
            x = getattr(self, "host", None)
            if x is None:
                x = pkg("workloads").softmax_input(self.rows, self.cols)
            t = x - x.max(axis=1, keepdims=True)
            self._subnormal = int(np.count_nonzero((t >= -103.28) & (t < -87.34)))
        return self._subnormal

    def config(self):
        return {"workload": "row_softmax", "rows": self.rows * self.world, "rows_per_gpu": self.rows,
                "cols": self.cols, "inputs": "N(0,16), 1% set to -100, seeded",
                "operand_sets": "2, alternating per step (nothing carried in L2 between steps)",
                "exp_args_in_subnormal_range": self.subnormal_exp_args(),
                "l2": "inputs larger than L2", "parallelism": f"dp{self.world} (rows per GPU)"}


class Add(Workload):
    name, unit, bound, phase = "add", "GB/s", "hbm", "pointwise"
    kernels_per_step = 1
    profile = "pointwise_add_2e24"

    def __init__(self, rank, world, n=1 << 24):
        super().__init__(rank, world)
        self.n = n

    def work(self):
        return 3.0 * 4 * self.n

    def setup(self, ctx, torch):
        a, b = pkg("workloads").add_inputs(self.n)
        self.host = (a, b)
        self.prog = pkg("runtime").make_program(2, [("add", 0, 1, 0, 0.0)], 2)
        self.ctx = ctx
        # Two copies of the operands, used alternately: a step's 201 MB were
        # last touched two steps earlier, with 201 MB in between, so nothing
        # of them is left in the 126 MB L2 and every step streams from HBM.
        self.sets = []
        for _ in range(2):
            da, db = torch.from_numpy(a).cuda(), torch.from_numpy(b).cuda()
            dc = torch.empty_like(da)
            call = ctx.pointwise_call(self.prog, [da.data_ptr(), db.data_ptr()], dc.data_ptr(), self.n)
            self.sets.append((da, db, dc, call))
        self.i = 0

    def step(self):
        self.sets[self.i][3]()
        self.i ^= 1

    def e2e_setup(self, session):
        self.session = session
        self.pa, self.pb, self.pc = (session.pinned((self.n,)) for _ in range(3))
        self.pa[...] = self.host[0]
        self.pb[...] = self.host[1]
        self.e2e_bytes = (2 * self.pa.nbytes, self.pc.nbytes)

    def e2e_step(self):
        self.session.pointwise_host(self.prog, [self.pa, self.pb], self.pc)

    def cpu_once(self, rows):
        refs = importlib.import_module("oracle.refs")
        a, b = self.host
        refs.pointwise("add", a[:rows], b[:rows])
        return 3.0 * 4 * rows, f"float64 NumPy a+b over {rows} elements"

    default_rows = 1 << 24
    reference_rows = 1 << 22

    def config(self):
        return {"workload": "pointwise_add", "n": self.n * self.world, "n_per_gpu": self.n,
                "operand_sets": "2, alternating per step (nothing carried in L2 between steps)",
                "inputs": "a,b ~ U[-1,1] seeded", "l2": "inputs larger than L2",
                "parallelism": f"dp{self.world} (contiguous ranges per GPU)"}


class Attention(Workload):
    name, unit, bound, phase = "attention", "TFLOP/s", "tensor", "flash"
    profile = "attention_tf32x3_64x2048x128"

    def __init__(self, rank, world, bh=64, seq=2048, d=128):
        super().__init__(rank, world)
        self.bh, self.seq, self.d = bh, seq, d

    def work(self):
        return 4.0 * self.bh * self.seq * self.seq * self.d

    def dominant_work(self):
        # the fused kernel runs both contractions, three TF32 products each
        return 3.0 * self.work()

    def setup(self, ctx, torch):
        q, k, v = pkg("workloads").attention_inputs(self.bh, self.seq, self.d)
        if self.rank:
            q = np.random.default_rng(3001 + 7919 * self.rank).standard_normal(q.shape).astype(np.float32)
        self.host = (q, k, v)
        self.dq, self.dk, self.dv = (torch.from_numpy(t).cuda() for t in (q, k, v))
        self.do = torch.empty_like(self.dq)
        self.ctx = ctx
        self.call = ctx.attention_call(self.dq.data_ptr(), self.dk.data_ptr(), self.dv.data_ptr(),
                                       self.do.data_ptr(), self.bh, self.seq, self.seq, self.d, self.d)

    def step(self):
        self.call()

    def e2e_setup(self, session):
        self.session = session
        self.pin = [session.pinned(t.shape) for t in self.host]
        for p, t in zip(self.pin, self.host):
            p[...] = t
        self.pout = session.pinned(self.host[0].shape)
        self.e2e_bytes = (sum(t.nbytes for t in self.host), self.pout.nbytes)

    def e2e_step(self):
        self.session.attention_host(*self.pin, self.pout)

    def cpu_once(self, rows):
        refs = importlib.import_module("oracle.refs")
        q, k, v = self.host
        heads = max(1, rows)
        refs.attention_batched(q[:heads], k[:heads], v[:heads])
        return 4.0 * heads * self.seq * self.seq * self.d, f"float64 NumPy attention of {heads} head(s) (S {self.seq}, D {self.d})"

    default_rows = 2
    reference_rows = 1

    def config(self):
        return {"workload": "attention_3xtf32", "batch_heads": self.bh * self.world, "batch_heads_per_gpu": self.bh,
                "seq": self.seq, "head_dim": self.d, "scale": "1/sqrt(128)", "inputs": "Q,K,V ~ N(0,1) seeded",
                "l2": "inputs larger than L2", "parallelism": f"dp{self.world} (batch*heads per GPU)"}


def make_workload(name, rank, world):
    if name == "attention":
        return Attention(rank, world)
    if name == "gemm":
        return Gemm(rank, world)
    if name == "ragged":
        w = Gemm(rank, world, 4097, 1000, 777, ragged=True)
        w.profile = "gemm_tf32x3_ragged"
        return w
    if name == "softmax":
        return Softmax(rank, world)
    if name == "add":
        return Add(rank, world)
    raise SystemExit(f"unknown workload {name}")


def scale(unit: str) -> float:
    return 1e12 if unit == "TFLOP/s" else 1e9


# --------------------------------------------------------------------------- clocks
class ClockSampler:
    """nvidia-smi clock / throttle-reason samples while the timed region runs."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, device: int):
        self.device, self.proc, self.path = device, None, None

    def start(self):
        try:
            fd, self.path = tempfile.mkstemp(prefix="clocks-", suffix=".csv")
            os.close(fd)
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.device), f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "50", "-f", self.path], stdout=subprocess.DEVNULL, stderr=subprocess.DEVNULL)
        except (OSError, FileNotFoundError):
            self.proc = None

    def stop(self) -> dict:
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "samples": 0, "note": "nvidia-smi unavailable"}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        rows = []
        for line in Path(self.path).read_text().splitlines():
            parts = [p.strip() for p in line.split(",")]
            if len(parts) >= 9:
                rows.append(parts)
        os.unlink(self.path)
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in rows for i in range(4) if r[5 + i].lower().startswith("active")})

        def num(v):
            try:
                return float(v)
            except ValueError:
                return None
        sm = [num(r[1]) for r in rows if num(r[1]) is not None]
        mx = [num(r[2]) for r in rows if num(r[2]) is not None]
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": reasons, "samples": len(rows)}


# --------------------------------------------------------------------------- arms
def init_dist():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return rank, local, world


def strong_scaling_gemm(ctx, torch, dist, rank, world, barrier, max_over_ranks, steps=10, warmup=3) -> dict:
    """One 4096^3 GEMM split by rows of A over the ranks (mgpu.sharded_gemm):
    NCCL broadcasts B from rank 0, each rank multiplies its row slab with the
    C-ABI GEMM, NCCL all-gathers C.  Device-timed with CUDA events around the
    whole call, max over ranks."""
    mgpu, workloads = pkg("mgpu"), pkg("workloads")
    m = n = k = 4096
    a, b = workloads.gemm_inputs(m, n, k)
    shard = mgpu.partition(m, world, rank, align=128)
    a_rows = torch.from_numpy(a[shard.start:shard.start + shard.count]).cuda()
    b_dev = torch.from_numpy(b).cuda() if rank == 0 else torch.empty((k, n), device="cuda")

    def compute(a_part, b_full):
        c_part = torch.empty((a_part.shape[0], n), device="cuda")
        ctx.gemm(a_part.data_ptr(), b_full.data_ptr(), c_part.data_ptr(), a_part.shape[0], n, k)
        return c_part

    for _ in range(warmup):
        mgpu.sharded_gemm(a_rows, b_dev, m, rank, world, compute, torch, device="cuda")
    barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(steps):
        c = mgpu.sharded_gemm(a_rows, b_dev, m, rank, world, compute, torch, device="cuda")
    e1.record()
    barrier()
    ms = max_over_ranks(e0.elapsed_time(e1)) / steps
    # size-independent check of the gathered C: its column sums equal (1^T A) B
    col = c.double().sum(dim=0).cpu().numpy()
    want = a.astype(np.float64).sum(axis=0) @ b.astype(np.float64)
    rel = float(np.max(np.abs(col - want)) / np.max(np.abs(want)))
    return {"value": round(2.0 * m * n * k / (ms / 1e3) / 1e12, 3), "unit": "TFLOP/s", "ms_per_gemm": round(ms, 4),
            "n_gpus": world, "steps": steps, "problem": "one 4096x4096x4096 GEMM (strong scaling)",
            "collectives": "NCCL broadcast of B (64 MiB) from rank 0, all_gather of C row slabs (64 MiB)",
            "column_sum_rel_err": rel}


def run_ours(args) -> dict | None:
    import torch
    rank, local, world = init_dist()
    torch.cuda.set_device(local)
    dist = None
    if world > 1:
        import torch.distributed as dist
        # NCCL prints its version on stdout while the communicator comes up;
        # stdout must carry only the JSON line, so send that to stderr.
        with stdout_to_stderr():
            pkg("mgpu").init_from_env("nccl", timeout_s=120)
            dist.barrier()
    runtime, api = pkg("runtime"), pkg("api")
    ctx = runtime.Context(local)
    w = make_workload(args.workload, rank, world)
    w.setup(ctx, torch)

    def barrier():
        torch.cuda.synchronize()
        if dist is not None:
            dist.barrier()
        torch.cuda.synchronize()

    def max_over_ranks(x: float) -> float:
        if dist is None:
            return x
        t = torch.tensor([x], dtype=torch.float64, device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    for _ in range(args.warmup):
        w.step()
    ctx.sync()
    # --- device-resident timed region ------------------------------------------
    sampler = ClockSampler(local)
    sampler.start()
    time.sleep(0.3)
    ctx.timing_reset()
    # The dominant kernel is timed with CUDA events on every TIMING_EVERY-th
    # step of the timed region: an event pair between two kernels costs a few
    # microseconds of idle GPU front end, which would inflate a 40-us step.
    barrier()
    launches_before = ctx.kernel_launches()
    start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record()
    for i in range(args.steps):
        sampled = i % TIMING_EVERY == 0
        if sampled:
            ctx.timing(True, phases=[w.phase])
        w.step()
        if sampled:
            ctx.timing(False)
    stop.record()
    launches = ctx.kernel_launches() - launches_before
    barrier()
    clocks = sampler.stop()
    ctx.sync()  # surfaces a device-side error status
    ms = max_over_ranks(start.elapsed_time(stop))
    ctx.timing(False)
    dom_ms, dom_launches = ctx.timing_read(w.phase)
    dom_ms = max_over_ranks(dom_ms)
    if w.kernels_per_step == 1:
        # One kernel per step: its average launch duration is the timed
        # region's event time over its launches (back to back, gaps included);
        # a single bracketed launch would also count the event's launch latency.
        dom_ms, dom_launches = ms, launches
        launch_basis = "timed region / launches (one kernel per step)"
    else:
        launch_basis = f"CUDA event pair around the kernel on 1 in {TIMING_EVERY} steps of the timed region"
    # --- end-to-end through host arrays ------------------------------------------
    session = api.Session(local)
    w.e2e_setup(session)
    e2e_steps = max(3, min(args.steps, 20))
    for _ in range(2):
        w.e2e_step()
    session.sync()
    barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(e2e_steps):
        w.e2e_step()
    e1.record()
    session.sync()
    barrier()
    e2e_ms = max_over_ranks(e0.elapsed_time(e1))
    # --- strong scaling of one 4096^3 GEMM over NCCL (multi-GPU GEMM runs) ---------
    strong = None
    if world > 1 and isinstance(w, Gemm) and not w.ragged:
        strong = strong_scaling_gemm(ctx, torch, dist, rank, world, barrier, max_over_ranks)
    # --- report ------------------------------------------------------------------
    result = None
    if rank == 0:
        peaks, basis = measured_peaks()
        value = world * w.work() * args.steps / (ms / 1e3) / scale(w.unit)
        avg_launch_s = dom_ms / 1e3 / max(1, dom_launches)
        if w.bound == "tensor":
            achieved = w.dominant_work() / avg_launch_s / 1e12
            # A run whose SM clock the 1 kW power cap held below 90 % of its
            # maximum is compared with the sustained GEMM peak (measured the
            # same way, clocks settled under the cap); otherwise the burst peak.
            capped = (clocks.get("sm_mhz") or 0) < 0.9 * (clocks.get("sm_max_mhz") or 0)
            sustained = capped and "bf16_tflops_sustained" in peaks
            peak = (peaks["bf16_tflops_sustained"] if sustained else peaks["bf16_tflops"]) / 2.0
            peak_note = (f"{basis} bf16 dense TF/s / 2 = TF32 dense rate ("
                         + (f"sustained: SM clock {clocks.get('sm_mhz')} of {clocks.get('sm_max_mhz')} MHz under "
                            f"the power cap" if sustained else "burst") + ")")
            unit = "TFLOP/s"
        else:
            achieved = w.dominant_work() / avg_launch_s / 1e9
            peak = peaks["hbm_gbs"]
            peak_note = f"{basis} HBM copy GB/s"
            unit = "GB/s"
        cpu = None
        if world == 1 and not args.no_cpu:
            v, sample = w.cpu_sample()
            cpu = {"value": round(v, 4), "unit": w.unit, "cores": os.cpu_count(), "kind": "port",
                   "sample": sample + " (oracle/refs.py float64 equations, NumPy/BLAS threads = all cores)"}
            cpu.update(w.cpu_extras())
        result = {
            "metric": METRIC, "value": round(value, 3), "unit": w.unit, "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(ms / args.steps, 5), "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "f32 (3xtf32 tensor)" if w.bound == "tensor" else "f32",
            "data": "synthetic (seeded, distributions of the BASELINE configs)",
            "config": w.config(),
            "e2e": {"value": round(world * w.work() * e2e_steps / (e2e_ms / 1e3) / scale(w.unit), 3), "unit": w.unit,
                    "h2d_bytes_per_step": int(w.e2e_bytes[0]), "d2h_bytes_per_step": int(w.e2e_bytes[1]),
                    "steps": e2e_steps, "api": "api.Session pipelined host-array calls (b2k_*_host: slabbed copy-in, kernels and copy-out overlapped)"},
            "roofline": {"bound": w.bound, "achieved": round(achieved, 2), "peak": round(peak, 2), "unit": unit,
                         "frac": round(achieved / peak, 4), "traffic": profile_traffic(w.profile),
                         "kernel": w.phase, "launch_ms": round(avg_launch_s * 1e3, 5), "launch_timing": launch_basis,
                         "peak_basis": peak_note},
            "cpu_baseline": cpu,
            "clocks": clocks,
            **({"strong_scaling_nccl": strong} if strong else {}),
            "gpu_launches": launches,
        }
    session.close()
    ctx.close()
    if dist is not None:
        dist.barrier()
        dist.destroy_process_group()
    return result


def run_reference(args) -> dict | None:
    rank, local, world = init_dist()
    if rank != 0:
        return None
    w = make_workload(args.workload, 0, 1)
    # host inputs only (no device)
    if isinstance(w, Gemm):
        w.host = w.inputs()
    elif isinstance(w, Attention):
        w.host = pkg("workloads").attention_inputs(w.bh, w.seq, w.d)
    elif isinstance(w, Softmax):
        w.host = pkg("workloads").softmax_input(w.rows, w.cols)
    else:
        w.host = pkg("workloads").add_inputs(w.n)
    # one bounded sample per step: a few tens of ms, so even thousands of
    # steps end within minutes
    for _ in range(args.warmup):
        w.cpu_sample(max_seconds=0.0, rows=w.reference_rows)
    values, samples = [], ""
    t0 = time.perf_counter()
    for _ in range(args.steps):
        v, samples = w.cpu_sample(max_seconds=0.0, rows=w.reference_rows)
        values.append(v)
    dt = time.perf_counter() - t0
    value = statistics.mean(values)
    return {"metric": METRIC, "value": round(value, 4), "unit": w.unit, "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(dt / args.steps * 1e3, 3), "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "f64", "data": "synthetic", "impl": "reference",
            "config": w.config(),
            "cpu_baseline": {"value": round(value, 4), "unit": w.unit, "cores": os.cpu_count(), "kind": "port",
                             "sample": samples + " per step (oracle/refs.py float64 equations of "
                                                 "tools/research_cases.py:74-103)", **w.cpu_extras()},
            "e2e": {"value": round(value, 4), "unit": w.unit, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}


def main():
    parser = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    parser.add_argument("--gpus", type=int, default=1)
    parser.add_argument("--steps", type=int, default=None)
    parser.add_argument("--warmup", type=int, default=5)
    parser.add_argument("--workload", default="gemm", choices=["gemm", "softmax", "add", "ragged", "attention"])
    parser.add_argument("--impl", default="ours", choices=["ours", "reference"])
    parser.add_argument("--no-cpu", action="store_true", help="skip the CPU baseline sample")
    args = parser.parse_args()
    if args.steps is None:
        args.steps = {"gemm": 1500, "ragged": 20000, "softmax": 20000, "add": 20000, "attention": 500}[args.workload]
        if args.impl == "reference":
            args.steps = 20
    args.warmup = max(3, args.warmup) if args.impl == "ours" else args.warmup
    result = run_reference(args) if args.impl == "reference" else run_ours(args)
    if result is not None:
        print(json.dumps(result), flush=True)


if __name__ == "__main__":
    main()
