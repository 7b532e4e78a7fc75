#!/usr/bin/env python3
"""Benchmark of the B200 backend's hot path (one JSON line on rank 0).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--workload gemm|softmax|add|ragged|attention]
                    [--impl ours|reference] [--only] [--no-graph]

A step is one pass of the hot path over one batch of synthetic input, the
BASELINE configurations:

* ``gemm`` (default, the headline) -- the 4096^3 FP32 GEMM as 3xTF32 on
  tcgen05 (operand split + tensor-core kernel), TFLOP/s of useful 2*M*N*K work;
* ``softmax`` -- row softmax of 4096 x 8192 FP32, GB/s of one read + one write;
* ``add`` -- c = a + b over 2^24 FP32, GB/s of two reads + one write;
* ``ragged`` -- relu(A B^T + bias), 4097 x 1000 x 777, TFLOP/s;
* ``attention`` -- softmax(Q K^T / sqrt(128)) V over 4 x 16 heads, S 2048,
  D 128, both contractions 3xTF32, TFLOP/s of useful 4*BH*S*S*D work.

The one-kernel workloads (softmax, add) issue their K timed steps as one
CUDA graph of the same library calls, replayed once (``step_issue`` in the
line; ``--no-graph`` issues every step from Python instead).

The line's top-level keys describe the selected workload (``--workload``,
gemm by default); unless ``--only`` is given, a ``workloads`` object carries
the same record (value, roofline, CPU baseline, end to end, clocks) for the
other four configurations, each timed in its own region of the same run,
and the GEMM and attention records carry a ``sustained`` leg: the same step
repeated for at least two seconds with its own clock samples.

With N > 1 (torchrun, one rank per GPU) ONE problem of the BASELINE size is
partitioned over the ranks (rows of A, rows of the softmax, element ranges,
batch*heads; ``mgpu.partition``) with every rank's shard already in its HBM:
strong scaling, ``value`` = the whole problem's work over the max-over-ranks
device time.  ``nccl_e2e`` repeats the partitioned step with its collectives
(B broadcast from rank 0, all-gather of the output slabs) through the
library's multi-GPU driver (``b2k_mgpu_*``, its own NCCL communicator), and ``weak`` gives
the replica figure (every rank the whole problem).  ``e2e`` is the step
through the public host-array API (``api.Session``, the ``b2k_*_host``
calls) with every rank's inputs copied in from page-locked host memory and
its outputs copied out, every step.  ``--impl reference`` times the
reference's CPU evaluation of the same workloads -- its float64 NumPy
equations (tools/research_cases.py:74-103, suite.py:192-234), restated in
``oracle/refs.py`` -- on the host cores, one full evaluation per step.
"""
from __future__ import annotations

import argparse
import contextlib
import importlib
import json
import math
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
WORKLOADS = ("gemm", "softmax", "add", "ragged", "attention")


def pkg(name):
    return importlib.import_module(f"{PKG}.{name}")


def oracle_refs():
    return importlib.import_module("oracle.refs")


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


def scale(unit: str) -> float:
    return 1e12 if unit == "TFLOP/s" else 1e9


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


# --------------------------------------------------------------------------- workloads
class Workload:
    """One BASELINE configuration, partitioned over `world` ranks (this rank's
    shard = `self.shard`), or whole on every rank when `replica` is set."""

    name = unit = bound = phase = profile = ""
    kernels_per_step = 1      # kernels of the hot path per step
    align = 1                 # shard granularity (units)
    steps_default = 2000      # timed steps of a secondary record
    cpu_seconds = 6.0         # CPU baseline sample length

    def __init__(self, rank: int, world: int, replica: bool = False):
        self.rank, self.world, self.replica = rank, world, replica
        mgpu = pkg("mgpu")
        self.shard = (mgpu.Shard(0, self.units()) if replica or world == 1
                      else mgpu.partition(self.units(), world, rank, self.align))

    # the partitioned axis: its extent and the work per unit
    def units(self) -> int:
        raise NotImplementedError

    def work_per_unit(self) -> float:
        raise NotImplementedError

    def work_total(self) -> float:
        """Work of all ranks per step: the whole problem, or one whole problem
        per rank for replicas (an emulated shard: that shard's work)."""
        if getattr(self, "emulated", False):
            return self.work_shard()
        return self.work_per_unit() * self.units() * (self.world if self.replica else 1)

    def work_shard(self) -> float:
        return self.work_per_unit() * self.shard.count

    def dominant_work(self) -> float:
        """Algorithmic work of one launch of the dominant kernel on this rank."""
        return self.work_shard()

    def operand_bytes(self) -> int:
        """Bytes of this rank's inputs and outputs (one operand set)."""
        raise NotImplementedError

    def operand_sets(self) -> int:
        """Operand copies rotated step by step (at least two): the data a step
        reads was last touched at least an L2's worth of traffic earlier.
        With one copy, part of a step's inputs survives in L2 for the next
        step even when the inputs are larger than L2 (the 201 MB add then
        reads at 1.1x the HBM copy rate)."""
        size = max(1, self.operand_bytes())
        return max(2, min(8, math.ceil(L2_BYTES / size) + 1))

    def l2_note(self) -> str:
        sets = self.operand_sets()
        return (f"{sets} operand sets rotated per step ({self.operand_bytes() / 2**20:.0f} MiB each): a step's inputs "
                f"were last touched {(sets - 1) * self.operand_bytes() / 2**20:.0f} MiB of traffic earlier, at least "
                "the 126 MB L2")

    # device set-up and one step (kernels only, shard pre-placed)
    def setup(self, ctx, torch):
        self.ctx = ctx
        self.sets = [self.make_set(ctx, torch, i) for i in range(self.operand_sets())]
        self.i = 0

    def make_set(self, ctx, torch, i):
        raise NotImplementedError

    def step(self):
        self.sets[self.i]()
        self.i = (self.i + 1) % len(self.sets)

    # end to end through the public host-array API
    def e2e_setup(self, session):
        raise NotImplementedError

    def e2e_step(self):
        raise NotImplementedError

    # the partitioned step with its collectives (world > 1)
    def overlap_splits(self) -> int:
        """Pieces (row pieces, or B column panels for the GEMM) per rank in the
        collective step, each gathered while the next computes.  One: measured
        on two B200s, splitting made the step slower -- NCCL's collective
        kernels take SMs from the single-wave kernels they overlap -- GEMM
        560 -> 677 us with two panels, softmax 194 -> 248 us, add 116 -> 181 us
        with two pieces."""
        return 1

    def nccl_setup(self, ctx, torch, group):
        raise NotImplementedError

    def nccl_step(self):
        raise NotImplementedError

    # CPU baseline: the oracle's float64 equations on the whole problem
    def host_inputs(self):
        raise NotImplementedError

    def cpu_once(self) -> tuple[float, str]:
        """One evaluation; returns (work units done, description)."""
        raise NotImplementedError

    def cpu_sample(self, seconds: float | None = None) -> tuple[float, str]:
        seconds = self.cpu_seconds if seconds is None else seconds
        done, work, t0 = 0, 0.0, time.perf_counter()
        while True:
            units, what = self.cpu_once()
            work += units
            done += 1
            if time.perf_counter() - t0 >= seconds:
                break
        dt = time.perf_counter() - t0
        return work / dt / scale(self.unit), f"{done} x {what}"

    def cpu_extras(self) -> dict:
        return {}

    def config(self) -> dict:
        raise NotImplementedError

    def parallelism(self, axis: str) -> str:
        if getattr(self, "emulated", False):
            return (f"1 GPU running rank 0's shard of a {self.world}-way partition by {axis} "
                    f"({self.shard.count} of {self.units()}); value = that shard's work")
        if self.world == 1:
            return "1 GPU"
        if self.replica:
            return f"{self.world} replicas (every rank the whole problem)"
        return f"{self.world} GPUs, one problem partitioned by {axis} (rank {self.rank}: {self.shard.count} of {self.units()})"


PLAN_SPLITS = {0: "pre-pass (A and B split before the tensor-core kernel)",
               1: "direct (A split inside the tensor-core kernel)",
               2: "transposed (B split inside the tensor-core kernel, C^T = B^T A^T)"}


class Gemm(Workload):
    name, unit, bound, phase = "gemm", "TFLOP/s", "tensor", "mma"
    kernels_per_step = 2  # operand split + tensor-core kernel (3 when K is chunk-split: + the fold)
    align = 128
    steps_default = 200
    cpu_seconds = 8.0

    def __init__(self, rank, world, replica=False, m=4096, n=4096, k=4096, ragged=False):
        self.m, self.n, self.k, self.ragged = m, n, k, ragged
        super().__init__(rank, world, replica)

    def units(self):
        return self.m

    def work_per_unit(self):
        return 2.0 * self.n * self.k

    def dominant_work(self):
        # the tensor core executes three TF32 products per useful one
        return 3.0 * self.work_shard()

    def host_inputs(self):
        if getattr(self, "_host", None) is None:
            w = pkg("workloads")
            if self.ragged:
                self._host = w.ragged_inputs(self.m, self.n, self.k)
            else:
                a, b = w.gemm_inputs(self.m, self.n, self.k)
                self._host = (a, b, None)
        return self._host

    def local(self):
        a, b, bias = self.host_inputs()
        return a[self.shard.start:self.shard.start + self.shard.count], b, bias

    def operand_bytes(self):
        a, b, bias = self.local()
        return a.nbytes + b.nbytes + 4 * a.shape[0] * self.n

    def make_set(self, ctx, torch, i):
        a, b, bias = self.local()
        da, db = torch.from_numpy(np.ascontiguousarray(a)).cuda(), torch.from_numpy(b).cuda()
        dbias = torch.from_numpy(bias).cuda() if bias is not None else None
        dc = torch.empty((a.shape[0], self.n), dtype=torch.float32, device="cuda")
        call = ctx.gemm_call(da.data_ptr(), db.data_ptr(), dc.data_ptr(), a.shape[0], self.n, self.k,
                             b_layout=1 if self.ragged else 0,
                             bias=dbias.data_ptr() if dbias is not None else 0, relu=self.ragged)
        call.keep = (da, db, dbias, dc)
        if getattr(self, "plan", None) is None:
            # the library's own path decision for this rank's call (b2k_gemm_plan)
            p = pkg("runtime").gemm_plan(ctx.sm_count, a.shape[0], self.n, self.k, a=da.data_ptr(), b=db.data_ptr(),
                                         b_layout=1 if self.ragged else 0)
            self.plan = {"split": PLAN_SPLITS[p["split_mode"]], "tile_width": p["tile_width"],
                         "k_chunk_split": p["chunk_split"], "k_chunks": p["chunks"]}
        return call

    def e2e_setup(self, session):
        a, b, bias = self.local()
        self.session = session
        self.pa, self.pb = session.pinned(a.shape), session.pinned(b.shape)
        self.pa[...] = a
        self.pb[...] = b
        self.pbias = None
        if bias is not None:
            self.pbias = session.pinned(bias.shape)
            self.pbias[...] = bias
        self.pc = session.pinned((a.shape[0], self.n))
        self.e2e_bytes = (a.nbytes + b.nbytes + (bias.nbytes if bias is not None else 0), self.pc.nbytes)

    def e2e_step(self):
        self.session.gemm_host(self.pa, self.pb, self.pc, b_layout="nk" if self.ragged else "kn",
                               bias=self.pbias, relu=self.ragged)

    def nccl_setup(self, ctx, torch, group):
        a, b, bias = self.local()
        self.torch, self.group = torch, group
        self.n_a = torch.from_numpy(np.ascontiguousarray(a)).cuda()
        self.n_b = torch.from_numpy(np.ascontiguousarray(b)).cuda() if self.rank == 0 else None
        self.n_bias = torch.from_numpy(bias).cuda() if bias is not None else None
        self.n_c = torch.empty((self.m, self.n), device="cuda")
        # the ragged GEMM's 1000 columns stay one panel (500-column panels
        # would not fill the GPU)
        self.panels = 1 if self.ragged else self.overlap_splits()
        self.nccl_note = (f"b2k_mgpu_gemm_tf32x3: NCCL broadcast of B ({b.nbytes / 2**20:.0f} MiB) from rank 0 in "
                          f"{self.panels} column panel(s), local GEMM per panel, all-gather of C "
                          f"({self.m * self.n * 4 / 2**20:.0f} MiB); panel p+1's broadcast and panel p's gather "
                          "overlap the GEMMs")

    def nccl_step(self):
        self.group.gemm(self.n_a.data_ptr(), self.n_b.data_ptr() if self.n_b is not None else 0,
                        self.n_c.data_ptr(), self.m, self.n, self.k, align=self.align,
                        b_layout=1 if self.ragged else 0,
                        bias=self.n_bias.data_ptr() if self.n_bias is not None else 0, relu=self.ragged,
                        panels=self.panels)
        return self.n_c

    def cpu_once(self):
        refs = oracle_refs()
        a, b, bias = self.host_inputs()
        if self.ragged:
            refs.matmul_bias_relu(a, b, bias)
        else:
            refs.matmul(a, b)
        return 2.0 * self.m * self.n * self.k, (f"float64 NumPy evaluation of the whole {self.m}x{self.n}x{self.k} "
                                                "GEMM" + (" + bias + ReLU" if self.ragged else ""))

    def cpu_extras(self):
        extras = {}
        with contextlib.suppress(ImportError):
            from threadpoolctl import threadpool_limits
            refs = oracle_refs()
            a, b, bias = self.host_inputs()
            rows = 256
            b64 = refs._f64(b).T.copy() if self.ragged else refs._f64(b)
            with threadpool_limits(limits=1):
                reps, t0 = 0, time.perf_counter()
                while reps < 2 or time.perf_counter() - t0 < 1.5:
                    refs._f64(a[:rows]) @ b64
                    reps += 1
                dt = (time.perf_counter() - t0) / reps
            extras["single_core"] = {"value": round(2.0 * rows * self.n * self.k / dt / 1e12, 5), "unit": self.unit,
                                     "sample": f"{reps} x float64 matmul of a {rows}-row slab of A, BLAS on 1 thread"}
        # tf32_emitter.py:64-96's model (per-8-K atom, three FP32 accumulators),
        # restated in oracle/tf32.py, on a 256^3 GEMM: its cost is linear in flop.
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

    @property
    def profile(self):
        """The committed ncu summary of this rank's dominant kernel shape."""
        if self.shard.count == self.m:
            return "gemm_tf32x3_ragged" if self.ragged else "gemm_tf32x3_4096"
        return f"gemm_tf32x3_shard_{self.shard.count}x{self.n}x{self.k}"

    def config(self):
        return {"workload": "ragged_gemm_bias_relu" if self.ragged else "gemm_3xtf32",
                "m": self.m, "n": self.n, "k": self.k, "m_this_rank": self.shard.count,
                "b_layout": "n_k (transposed)" if self.ragged else "k_n",
                "epilogue": "bias+relu" if self.ragged else "copy",
                "inputs": "A,B ~ N(0,1) seeded" if self.ragged else "A,B ~ U[-1,1] seeded",
                "l2": self.l2_note(), "parallelism": self.parallelism("rows of A (B replicated)")}


class Softmax(Workload):
    name, unit, bound, phase = "softmax", "GB/s", "hbm", "softmax"
    profile = "row_softmax_4096x8192"
    steps_default = 2000

    def __init__(self, rank, world, replica=False, rows=4096, cols=8192):
        self.rows, self.cols = rows, cols
        super().__init__(rank, world, replica)

    def units(self):
        return self.rows

    def work_per_unit(self):
        return 2.0 * 4 * self.cols

    def host_inputs(self):
        if getattr(self, "_host", None) is None:
            self._host = pkg("workloads").softmax_input(self.rows, self.cols)
        return self._host

    def local(self):
        return self.host_inputs()[self.shard.start:self.shard.start + self.shard.count]

    def operand_bytes(self):
        return 2 * self.local().nbytes

    def make_set(self, ctx, torch, i):
        x = self.local()
        dx = torch.from_numpy(np.ascontiguousarray(x)).cuda()
        dy = torch.empty_like(dx)
        call = ctx.row_softmax_call(dx.data_ptr(), dy.data_ptr(), x.shape[0], self.cols)
        call.keep = (dx, dy)
        return call

    def e2e_setup(self, session):
        x = self.local()
        self.session = session
        self.px = session.pinned(x.shape)
        self.px[...] = x
        self.py = session.pinned(x.shape)
        self.e2e_bytes = (self.px.nbytes, self.py.nbytes)

    def e2e_step(self):
        self.session.row_softmax_host(self.px, self.py)

    def nccl_setup(self, ctx, torch, group):
        self.torch, self.group = torch, group
        self.n_x = torch.from_numpy(np.ascontiguousarray(self.local())).cuda()
        self.n_y = torch.empty((self.rows, self.cols), device="cuda")
        self.nccl_note = (f"b2k_mgpu_row_softmax_f32: local softmax, all-gather of the output rows ({self.rows * self.cols * 4 / 2**20:.0f} MiB) "
                          f"in {self.overlap_splits()} piece(s) per rank, each gathered while the next computes")

    def nccl_step(self):
        self.group.row_softmax(self.n_x.data_ptr(), self.n_y.data_ptr(), self.rows, self.cols,
                               pieces=self.overlap_splits())
        return self.n_y

    def cpu_once(self):
        oracle_refs().softmax(self.host_inputs())
        return 2.0 * 4 * self.rows * self.cols, f"float64 NumPy stable softmax of the whole {self.rows}x{self.cols} matrix"

    def subnormal_exp_args(self) -> int:
        """How many exp arguments x - rowmax of this input give a subnormal
        FP32 result (arguments in [-103.28, -87.34]): the range the selective
        exponential exists for."""
        x = self.host_inputs()
        t = x - x.max(axis=1, keepdims=True)
        return int(np.count_nonzero((t >= -103.28) & (t < -87.34)))

    def config(self):
        return {"workload": "row_softmax", "rows": self.rows, "rows_this_rank": self.shard.count, "cols": self.cols,
                "inputs": "N(0,16), 1% set to -100, seeded", "exp_args_in_subnormal_range": self.subnormal_exp_args(),
                "l2": self.l2_note(), "parallelism": self.parallelism("rows")}


class Add(Workload):
    name, unit, bound, phase = "add", "GB/s", "hbm", "pointwise"
    profile = "pointwise_add_2e24"
    align = 4
    steps_default = 2000
    cpu_seconds = 4.0

    def __init__(self, rank, world, replica=False, n=1 << 24):
        self.n = n
        super().__init__(rank, world, replica)

    def units(self):
        return self.n

    def work_per_unit(self):
        return 3.0 * 4

    def host_inputs(self):
        if getattr(self, "_host", None) is None:
            self._host = pkg("workloads").add_inputs(self.n)
        return self._host

    def local(self):
        a, b = self.host_inputs()
        sl = slice(self.shard.start, self.shard.start + self.shard.count)
        return a[sl], b[sl]

    def operand_bytes(self):
        return 3 * self.local()[0].nbytes

    def program(self):
        if getattr(self, "_prog", None) is None:
            self._prog = pkg("runtime").make_program(2, [("add", 0, 1, 0, 0.0)], 2)
        return self._prog

    def make_set(self, ctx, torch, i):
        a, b = self.local()
        da, db = torch.from_numpy(np.ascontiguousarray(a)).cuda(), torch.from_numpy(np.ascontiguousarray(b)).cuda()
        dc = torch.empty_like(da)
        call = ctx.pointwise_call(self.program(), [da.data_ptr(), db.data_ptr()], dc.data_ptr(), a.size)
        call.keep_tensors = (da, db, dc)
        return call

    def e2e_setup(self, session):
        a, b = self.local()
        self.session = session
        self.pa, self.pb, self.pc = (session.pinned(a.shape) for _ in range(3))
        self.pa[...] = a
        self.pb[...] = b
        self.e2e_bytes = (2 * self.pa.nbytes, self.pc.nbytes)

    def e2e_step(self):
        self.session.pointwise_host(self.program(), [self.pa, self.pb], self.pc)

    def nccl_setup(self, ctx, torch, group):
        self.torch, self.group = torch, group
        a, b = self.local()
        self.n_a, self.n_b = torch.from_numpy(np.ascontiguousarray(a)).cuda(), torch.from_numpy(np.ascontiguousarray(b)).cuda()
        self.n_c = torch.empty(self.n, device="cuda")
        self.nccl_note = (f"b2k_mgpu_pointwise_f32: local add, all-gather of c's element ranges ({self.n * 4 / 2**20:.0f} MiB) in "
                          f"{self.overlap_splits()} piece(s) per rank, each gathered while the next computes")

    def nccl_step(self):
        self.group.pointwise(self.program(), [self.n_a.data_ptr(), self.n_b.data_ptr()], self.n_c.data_ptr(),
                             self.n, align=self.align, pieces=self.overlap_splits())
        return self.n_c

    def cpu_once(self):
        a, b = self.host_inputs()
        oracle_refs().pointwise("add", a, b)
        return 3.0 * 4 * self.n, f"float64 NumPy a + b over all {self.n} elements"

    def config(self):
        return {"workload": "pointwise_add", "n": self.n, "n_this_rank": self.shard.count,
                "inputs": "a,b ~ U[-1,1] seeded", "l2": self.l2_note(),
                "parallelism": self.parallelism("contiguous element ranges")}


class Attention(Workload):
    name, unit, bound, phase = "attention", "TFLOP/s", "tensor", "flash"
    profile = "attention_tf32x3_64x2048x128"
    kernels_per_step = 3
    steps_default = 100
    cpu_heads = 8           # heads per CPU sample (one head is ~0.3 s of float64 BLAS)

    def overlap_splits(self) -> int:
        """Two pieces of heads at 2 and 4 GPUs (each still several waves of
        query tiles), one at 8: measured on two B200s, 494 -> 483 us."""
        return 2 if self.world in (2, 4) else 1

    def __init__(self, rank, world, replica=False, bh=64, seq=2048, d=128):
        self.bh, self.seq, self.d = bh, seq, d
        super().__init__(rank, world, replica)

    def units(self):
        return self.bh

    def work_per_unit(self):
        return 4.0 * self.seq * self.seq * self.d

    def dominant_work(self):
        # the fused kernel runs both contractions, three TF32 products each
        return 3.0 * self.work_shard()

    def host_inputs(self):
        if getattr(self, "_host", None) is None:
            self._host = pkg("workloads").attention_inputs(self.bh, self.seq, self.d)
        return self._host

    def local(self):
        sl = slice(self.shard.start, self.shard.start + self.shard.count)
        return tuple(t[sl] for t in self.host_inputs())

    def operand_bytes(self):
        return 4 * self.local()[0].nbytes

    def make_set(self, ctx, torch, i):
        q, k, v = self.local()
        dq, dk, dv = (torch.from_numpy(np.ascontiguousarray(t)).cuda() for t in (q, k, v))
        do = torch.empty_like(dq)
        call = ctx.attention_call(dq.data_ptr(), dk.data_ptr(), dv.data_ptr(), do.data_ptr(), q.shape[0], self.seq,
                                  self.seq, self.d, self.d)
        call.keep = (dq, dk, dv, do)
        return call

    def e2e_setup(self, session):
        q, k, v = self.local()
        self.session = session
        self.pin = [session.pinned(t.shape) for t in (q, k, v)]
        for p, t in zip(self.pin, (q, k, v)):
            p[...] = t
        self.pout = session.pinned(q.shape)
        self.e2e_bytes = (3 * q.nbytes, self.pout.nbytes)

    def e2e_step(self):
        self.session.attention_host(*self.pin, self.pout)

    def nccl_setup(self, ctx, torch, group):
        self.torch, self.group = torch, group
        self.n_in = [torch.from_numpy(np.ascontiguousarray(t)).cuda() for t in self.local()]
        self.n_o = torch.empty((self.bh, self.seq, self.d), device="cuda")
        self.nccl_note = (f"b2k_mgpu_attention_tf32x3: heads pre-sharded with Q, K and V (nothing broadcast), all-gather of O "
                          f"({self.bh * self.seq * self.d * 4 / 2**20:.0f} MiB) in {self.overlap_splits()} piece(s) per "
                          "rank, each gathered while the next computes")

    def nccl_step(self):
        q, k, v = self.n_in
        self.group.attention(q.data_ptr(), k.data_ptr(), v.data_ptr(), self.n_o.data_ptr(), self.bh, self.seq,
                             self.seq, self.d, self.d, pieces=self.overlap_splits())
        return self.n_o

    def cpu_once(self):
        q, k, v = self.host_inputs()
        h = self.cpu_heads
        oracle_refs().attention_batched(q[:h], k[:h], v[:h])
        return 4.0 * h * self.seq * self.seq * self.d, (f"float64 NumPy attention of {h} whole heads (S {self.seq}, "
                                                        f"D {self.d}) of the 64")

    def config(self):
        return {"workload": "attention_3xtf32", "batch_heads": self.bh, "heads_this_rank": self.shard.count,
                "seq": self.seq, "head_dim": self.d, "scale": "1/sqrt(128)", "inputs": "Q,K,V ~ N(0,1) seeded",
                "l2": self.l2_note(), "parallelism": self.parallelism("batch*heads")}


def make_workload(name, rank, world, replica=False):
    if name == "attention":
        return Attention(rank, world, replica)
    if name == "gemm":
        return Gemm(rank, world, replica)
    if name == "ragged":
        w = Gemm(rank, world, replica, 4097, 1000, 777, ragged=True)
        w.name, w.steps_default, w.cpu_seconds = "ragged", 2000, 4.0
        return w
    if name == "softmax":
        return Softmax(rank, world, replica)
    if name == "add":
        return Add(rank, world, replica)
    raise SystemExit(f"unknown workload {name}")


# --------------------------------------------------------------------------- clocks
class ClockSampler:
    """nvidia-smi clock / throttle-reason samples while a timed region runs."""

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
        pw = [num(r[3]) for r in rows if num(r[3]) is not None]
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": reasons, "samples": len(rows), "power_w_max": max(pw) if pw else None}


# --------------------------------------------------------------------------- our arm
def init_dist():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return rank, local, world


class Runner:
    """Per-process state of our arm: the context, the process group helpers."""

    TIMING_EVERY = 8  # steps per sampled launch of a multi-kernel step's dominant kernel

    def __init__(self, torch, dist, rank, local, world):
        self.torch, self.dist, self.rank, self.local, self.world = torch, dist, rank, local, world
        self.ctx = pkg("runtime").Context(local)
        self.peaks, self.peak_basis = measured_peaks()
        self.group = None
        self.use_graphs = True

    def native_group(self):
        """The library's own NCCL communicator (b2k_mgpu_*): rank 0 makes the
        rendezvous id, the process group hands it to every rank."""
        if self.group is None:
            rt, torch = pkg("runtime"), self.torch
            uid = torch.zeros(rt.MGPU_ID_BYTES, dtype=torch.uint8, device="cuda")
            if self.rank == 0:
                uid.copy_(torch.frombuffer(bytearray(rt.mgpu_unique_id()), dtype=torch.uint8))
            if self.dist is not None:
                self.dist.broadcast(uid, src=0)
            with stdout_to_stderr():  # NCCL may print its version while the communicator comes up
                self.group = rt.MultiGpu(self.ctx, self.world, self.rank, bytes(uid.cpu().numpy().tobytes()))
        return self.group

    def barrier(self):
        self.torch.cuda.synchronize()
        if self.dist is not None:
            self.dist.barrier()
        self.torch.cuda.synchronize()

    def max_over_ranks(self, x: float) -> float:
        if self.dist is None:
            return x
        t = self.torch.tensor([x], dtype=self.torch.float64, device="cuda")
        self.dist.all_reduce(t, op=self.dist.ReduceOp.MAX)
        return float(t.item())

    def event_pair(self):
        return (self.torch.cuda.Event(enable_timing=True), self.torch.cuda.Event(enable_timing=True))

    def capture(self, w: Workload, steps: int):
        """The `steps` steps of a one-kernel workload as one CUDA graph: the same
        bound library calls (same buffers, same operand-set rotation as the
        loop), issued on a stream being captured.  A call made from Python costs
        a few microseconds of host time, more than a whole step of a small
        shard (the 2^21-element add of an 8-way partition); replayed from a
        graph, the steps run back to back on the device.  Returns (graph,
        launches captured, None) or (None, 0, the reason capture failed)."""
        torch = self.torch
        try:
            side = torch.cuda.Stream()
            calls = [call.with_stream(side.cuda_stream) for call in w.sets]
            graph = torch.cuda.CUDAGraph()
            self.ctx.sync()
            before = self.ctx.kernel_launches()
            # thread-local capture: other threads (the process group's NCCL
            # watchdog) keep querying their events while this one captures
            with torch.cuda.graph(graph, stream=side, capture_error_mode="thread_local"):
                for i in range(steps):
                    calls[i % len(calls)]()
            launches = self.ctx.kernel_launches() - before
            graph.replay()  # untimed: uploads the graph, warms the kernels
            torch.cuda.synchronize()
            return graph, launches, None
        except Exception as exc:  # the loop is used instead, and the line says why
            torch.cuda.synchronize()
            return None, 0, f"{type(exc).__name__}: {exc}"

    def timed(self, w: Workload, steps: int, warmup: int, sample_dominant: bool = True) -> dict:
        """Warm-up, then EXACTLY `steps` steps between barriers; device time with
        CUDA events (max over ranks), clocks sampled during the region, and the
        dominant kernel's average launch time.  One-kernel workloads replay
        their steps from a CUDA graph (see `capture`)."""
        ctx = self.ctx
        for _ in range(warmup):
            w.step()
        ctx.sync()
        graph, graph_launches, graph_error = (None, 0, "the workload has several kernels per step")
        if w.kernels_per_step == 1 and self.use_graphs:
            graph, graph_launches, graph_error = self.capture(w, steps)
        sampler = ClockSampler(self.local)
        sampler.start()
        time.sleep(0.3)
        ctx.timing_reset()
        self.barrier()
        launches_before = ctx.kernel_launches()
        start, stop = self.event_pair()
        start.record()
        if graph is not None:
            graph.replay()
        else:
            for i in range(steps):
                sampled = sample_dominant and w.kernels_per_step > 1 and i % self.TIMING_EVERY == 0
                if sampled:
                    ctx.timing(True, phases=[w.phase])
                w.step()
                if sampled:
                    ctx.timing(False)
        stop.record()
        launches = graph_launches if graph is not None else ctx.kernel_launches() - launches_before
        self.barrier()
        clocks = sampler.stop()
        ctx.sync()  # surfaces a device-side error status
        ms = self.max_over_ranks(start.elapsed_time(stop))
        ctx.timing(False)
        if w.kernels_per_step == 1:
            # One kernel per step: its average launch duration is the timed
            # region's event time over its launches (back to back, gaps
            # included); a bracketed launch would add the events' own latency.
            dom_ms, dom_launches = ms, max(1, launches)
            basis = "timed region / launches (one kernel per step)"
        else:
            dom_ms, dom_launches = ctx.timing_read(w.phase)
            dom_ms = self.max_over_ranks(dom_ms)
            basis = f"CUDA event pair around the kernel on 1 in {self.TIMING_EVERY} steps of the timed region"
        issue = ("one CUDA graph of the timed steps' library calls, replayed once" if graph is not None
                 else f"one library call per step from Python ({graph_error})")
        return {"ms": ms, "steps": steps, "launches": launches, "clocks": clocks,
                "dom_ms": dom_ms / max(1, dom_launches), "dom_basis": basis, "issue": issue}

    def roofline(self, w: Workload, t: dict, sustained: bool = False) -> dict:
        peaks, basis = self.peaks, self.peak_basis
        launch_s = t["dom_ms"] / 1e3
        if w.bound == "tensor":
            achieved = w.dominant_work() / launch_s / 1e12
            # a long, power-capped region is compared with the sustained GEMM peak
            clocks = t["clocks"]
            capped = sustained or (clocks.get("sm_mhz") or 0) < 0.9 * (clocks.get("sm_max_mhz") or 0)
            use_sustained = capped and "bf16_tflops_sustained" in peaks
            peak = (peaks["bf16_tflops_sustained"] if use_sustained else peaks["bf16_tflops"]) / 2.0
            note = (f"{basis} bf16 dense TF/s / 2 = TF32 dense rate (" + ("sustained" if use_sustained else "burst")
                    + "); achieved counts the three TF32 products per useful one")
            unit = "TFLOP/s"
        else:
            achieved = w.dominant_work() / launch_s / 1e9
            peak = peaks["hbm_gbs"]
            note = f"{basis} HBM copy GB/s"
            unit = "GB/s"
        return {"bound": w.bound, "achieved": round(achieved, 2), "peak": round(peak, 2), "unit": unit,
                "frac": round(achieved / peak, 4), "traffic": profile_traffic(w.profile), "kernel": w.phase,
                "launch_ms": round(t["dom_ms"], 5), "launch_timing": t["dom_basis"], "peak_basis": note}

    def e2e(self, w: Workload, steps: int) -> dict:
        api = pkg("api")
        session = api.Session(self.local)
        try:
            w.e2e_setup(session)
            for _ in range(2):
                w.e2e_step()
            session.sync()
            self.barrier()
            e0, e1 = self.event_pair()
            e0.record()
            for _ in range(steps):
                w.e2e_step()
            e1.record()
            session.sync()
            self.barrier()
            ms = self.max_over_ranks(e0.elapsed_time(e1))
        finally:
            session.close()
        return {"value": round(w.work_total() * steps / (ms / 1e3) / scale(w.unit), 3), "unit": w.unit,
                "h2d_bytes_per_step": int(w.e2e_bytes[0]), "d2h_bytes_per_step": int(w.e2e_bytes[1]),
                "steps": steps, "ms_per_step": round(ms / steps, 4),
                "api": "api.Session pipelined host-array calls (b2k_*_host: slabbed copy-in, kernels and copy-out "
                       "overlapped)" + (", each rank its own shard" if self.world > 1 else "")}

    def nccl_e2e(self, w: Workload, steps: int = 10, warmup: int = 3) -> dict:
        """The partitioned step with its collectives, device-resident (max over
        ranks), through the library's multi-GPU driver (b2k_mgpu_*)."""
        group = self.native_group()
        w.nccl_setup(self.ctx, self.torch, group)
        for _ in range(warmup):
            out = w.nccl_step()
        group.sync(timeout_ms=120000)
        self.barrier()
        e0, e1 = self.event_pair()
        e0.record()
        for _ in range(steps):
            out = w.nccl_step()
        e1.record()
        group.sync(timeout_ms=120000)
        self.barrier()
        ms = self.max_over_ranks(e0.elapsed_time(e1))
        # size-independent check of the gathered output on every rank
        checksum = float(out.double().sum().item())
        return {"value": round(w.work_total() * steps / (ms / 1e3) / scale(w.unit), 3), "unit": w.unit,
                "ms_per_step": round(ms / steps, 4), "steps": steps, "collectives": w.nccl_note,
                "gathered_output_sum": checksum}

    def record(self, name: str, args, headline: bool) -> dict:
        """Every measurement of one workload; rank 0 gets the record."""
        torch = self.torch
        if self.world == 1 and args.shard_of > 1:
            w = make_workload(name, 0, args.shard_of)
            w.emulated = True
        else:
            w = make_workload(name, self.rank, self.world)
        w.setup(self.ctx, torch)
        steps = args.steps if headline else (args.sub_steps or w.steps_default)
        t = self.timed(w, steps, args.warmup)
        rec = {"metric": METRIC if headline else f"{w.name} {w.unit}",
               "value": round(w.work_total() * steps / (t["ms"] / 1e3) / scale(w.unit), 3), "unit": w.unit,
               "n_gpus": self.world, "steps": steps, "warmup": args.warmup, "ms_per_step": round(t["ms"] / steps, 5),
               "higher_is_better": True, "scaling": "strong" if self.world > 1 else "weak",
               "dtype": "f32 (3xtf32 tensor)" if w.bound == "tensor" else "f32",
               "config": w.config(), "roofline": self.roofline(w, t), "clocks": t["clocks"],
               "gpu_launches": t["launches"], "step_issue": t["issue"]}
        if getattr(w, "plan", None):
            rec["kernel_path"] = dict(w.plan, of="the device-resident calls of `value` (rank 0's shard)")
        if self.world > 1:
            rec["timing"] = ("kernels only, every rank's shard pre-placed in its HBM; time = max over ranks of each "
                             "rank's CUDA-event time")
        # sustained leg: the same step for >= 2 s (tensor-bound workloads, one GPU)
        if self.world == 1 and w.bound == "tensor" and not args.no_sustained:
            per_step_s = max(1e-6, t["ms"] / steps / 1e3)
            # the power cap slows a long region by up to ~20 %: aim well past 2 s
            s_steps = max(steps, int(math.ceil(2.5 / per_step_s)))
            ts = self.timed(w, s_steps, 0)
            rec["sustained"] = {"value": round(w.work_total() * s_steps / (ts["ms"] / 1e3) / scale(w.unit), 3),
                                "unit": w.unit, "steps": s_steps, "seconds": round(ts["ms"] / 1e3, 3),
                                "ms_per_step": round(ts["ms"] / s_steps, 5), "clocks": ts["clocks"],
                                "roofline": self.roofline(w, ts, sustained=True)}
        w.sets = []
        torch.cuda.empty_cache()
        # end to end through the public host-array API
        rec["e2e"] = self.e2e(w, max(3, min(steps, 20)))
        torch.cuda.empty_cache()
        if self.world > 1:
            rec["nccl_e2e"] = self.nccl_e2e(w)
            w.n_in = w.n_a = w.n_b = w.n_x = w.n_y = w.n_c = w.n_o = None
            torch.cuda.empty_cache()
            # replica figure: every rank the whole problem, no collective
            wr = make_workload(name, self.rank, self.world, replica=True)
            wr.setup(self.ctx, torch)
            tr = self.timed(wr, max(3, min(steps, 50)), args.warmup, sample_dominant=False)
            rec["weak"] = {"value": round(wr.work_total() * tr["steps"] / (tr["ms"] / 1e3) / scale(w.unit), 3),
                           "unit": w.unit, "ms_per_step": round(tr["ms"] / tr["steps"], 5), "steps": tr["steps"],
                           "problem": "every rank the whole BASELINE problem (replicas)"}
            wr.sets = []
            torch.cuda.empty_cache()
        if self.rank == 0 and self.world == 1 and not args.no_cpu and not getattr(w, "emulated", False):
            v, sample = w.cpu_sample()
            cpu = {"value": round(v, 4), "unit": w.unit, "cores": os.cpu_count(), "kind": "port",
                   "sample": sample + " (oracle/refs.py float64 equations, NumPy/BLAS threads = all cores)"}
            cpu.update(w.cpu_extras())
            rec["cpu_baseline"] = cpu
        else:
            rec["cpu_baseline"] = None
        return rec


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
    runner = Runner(torch, dist, rank, local, world)
    runner.use_graphs = not args.no_graph
    try:
        rec = runner.record(args.workload, args, headline=True)
        if not args.only:
            others = {}
            for name in WORKLOADS:
                if name != args.workload:
                    r = runner.record(name, args, headline=False)
                    r.pop("metric", None)
                    others[name] = r
            rec["workloads"] = others
        rec["vs_baseline"] = None
        rec["data"] = "synthetic (seeded, distributions of the BASELINE configs)"
    finally:
        if runner.group is not None:
            runner.group.close()
        runner.ctx.close()
        if dist is not None:
            dist.barrier()
            dist.destroy_process_group()
    if rank != 0:
        return None
    order = ["metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step", "higher_is_better", "scaling",
             "vs_baseline", "dtype", "data", "config"]
    return {**{k: rec[k] for k in order if k in rec}, **{k: v for k, v in rec.items() if k not in order}}


# --------------------------------------------------------------------------- reference arm
def reference_record(name: str, steps: int, warmup: int) -> dict:
    """The reference's CPU evaluation (float64 NumPy) of one workload, one full
    evaluation per step (attention: a stated number of whole heads)."""
    w = make_workload(name, 0, 1)
    w.host_inputs()
    for _ in range(warmup):
        w.cpu_once()
    t0 = time.perf_counter()
    work, what = 0.0, ""
    for _ in range(steps):
        units, what = w.cpu_once()
        work += units
    dt = time.perf_counter() - t0
    value = work / dt / scale(w.unit)
    return {"value": round(value, 4), "unit": w.unit, "steps": steps, "warmup": warmup,
            "ms_per_step": round(dt / steps * 1e3, 3), "config": w.config(),
            "cpu_baseline": {"value": round(value, 4), "unit": w.unit, "cores": os.cpu_count(), "kind": "port",
                             "sample": f"{what} per step (oracle/refs.py float64 equations of "
                                       "tools/research_cases.py:74-103 / suite.py:192-234, BLAS threads = all cores)"},
            "e2e": {"value": round(value, 4), "unit": w.unit, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}


def run_reference(args) -> dict | None:
    rank, _, world = init_dist()
    if rank != 0:
        return None
    rec = reference_record(args.workload, args.steps, args.warmup)
    out = {"metric": METRIC, "value": rec["value"], "unit": rec["unit"], "n_gpus": world, "steps": args.steps,
           "warmup": args.warmup, "ms_per_step": rec["ms_per_step"], "higher_is_better": True,
           "scaling": "strong" if world > 1 else "weak", "vs_baseline": None, "dtype": "f64", "data": "synthetic",
           "impl": "reference", "config": rec["config"], "cpu_baseline": rec["cpu_baseline"], "e2e": rec["e2e"]}
    if not args.only:
        out["workloads"] = {name: reference_record(name, 3, 1) for name in WORKLOADS if name != args.workload}
    return out


def main():
    parser = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    parser.add_argument("--gpus", type=int, default=1)
    parser.add_argument("--steps", type=int, default=None)
    parser.add_argument("--warmup", type=int, default=5)
    parser.add_argument("--workload", default="gemm", choices=list(WORKLOADS))
    parser.add_argument("--impl", default="ours", choices=["ours", "reference"])
    parser.add_argument("--only", action="store_true", help="measure the selected workload only")
    parser.add_argument("--sub-steps", type=int, default=None, help="timed steps of the other workloads' records")
    parser.add_argument("--no-cpu", action="store_true", help="skip the CPU baseline samples")
    parser.add_argument("--no-sustained", action="store_true", help="skip the >= 2 s sustained legs")
    parser.add_argument("--no-graph", action="store_true",
                        help="issue the one-kernel workloads' timed steps from Python instead of a CUDA graph")
    parser.add_argument("--shard-of", type=int, default=1,
                        help="on one GPU, time rank 0's shard of an N-way partition (profiling the multi-GPU shapes)")
    args = parser.parse_args()
    if args.steps is None:
        args.steps = 20 if args.impl == "reference" else make_workload(args.workload, 0, 1).steps_default
    args.warmup = max(3, args.warmup) if args.impl == "ours" else args.warmup
    result = run_reference(args) if args.impl == "reference" else run_ours(args)
    if result is not None:
        print(json.dumps(result), flush=True)


if __name__ == "__main__":
    main()
