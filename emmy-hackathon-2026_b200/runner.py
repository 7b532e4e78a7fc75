"""Run a recognised IR kernel (or multi-kernel pipeline) end to end on the GPU.

The reference's runner executes a launch request in a fresh worker
(tools/local_runner.py:246-342): inputs come from ``data`` or
``default_rng(seed).standard_normal(shape)`` (:152-158), outputs named in
``zero_outputs`` are zeroed before every launch (:320-322), every launch is
timed with CUDA events (:318-332) and the outputs are returned with a summary
(:160-165).  :func:`run` does the same through ``api.Session`` (device memory
and copies through the C ABI, no PyTorch) and the kernels recognised by
``frontend.compile_path``.
"""
from __future__ import annotations

import json
import statistics
from pathlib import Path

import numpy as np

from . import api, frontend, runtime

DTYPES = {"f32": np.float32}
PHASE_OF = {"pointwise": "pointwise", "row_softmax": "softmax", "matmul": "mma", "attention": "attention",
            "row_reduce": "rows", "row_norm": "rows", "axis_reduce": "rows"}


def array_for(arg) -> np.ndarray:
    """tools/local_runner.py:152-158."""
    dtype, shape = DTYPES[arg.get("dtype", "f32")], arg["shape"]
    if arg.get("output"):
        return np.zeros(shape, dtype=dtype)
    if "data" in arg:
        return np.ascontiguousarray(np.asarray(arg["data"], dtype=dtype).reshape(shape))
    return np.ascontiguousarray(np.random.default_rng(arg["seed"]).standard_normal(shape).astype(dtype))


def output_summary(array, arg, limit) -> dict:
    returned = min(array.size, limit)
    return {"shape": arg["shape"], "dtype": arg.get("dtype", "f32"), "sum": float(array.sum()),
            "values": array.reshape(-1)[:returned].tolist(), "truncated": returned < array.size}


class Pipeline:
    """The kernels of one case directory (``meta.json`` + ``*.ir.json``), recognised."""

    def __init__(self, folder):
        folder = Path(folder)
        if folder.is_file():
            folder = folder.parent
        self.folder = folder
        self.meta = json.loads((folder / "meta.json").read_text())
        irs = sorted(folder.glob("*.ir.json"))
        self.specs = []
        for kernel in self.meta["kernels"]:
            path = folder / f"{kernel['entry']}.ir.json"
            if not path.exists():
                if len(irs) != 1:
                    raise frontend.Unsupported(f"no IR file for entry {kernel['entry']!r}")
                path = irs[0]
            spec = frontend.compile_path(path)
            if spec.entry != kernel["entry"] or spec.node != kernel["node"]:
                raise frontend.Unsupported("IR file does not hold the metadata kernel")
            self.specs.append(spec)
        self.args = {}
        for kernel in self.meta["kernels"]:
            for arg in kernel["args"]:
                self.args.setdefault(arg["name"], arg)

    def run(self, session: api.Session, inputs: dict | None = None, warmup: int = 5, iters: int = 20,
            max_return: int = 4096) -> tuple[dict, dict]:
        """Returns (result record, {output name: array})."""
        host, device = {}, {}
        for name, arg in self.args.items():
            given = None if inputs is None else inputs.get(name)
            is_output = any(a["name"] == name and a.get("output") for k in self.meta["kernels"] for a in k["args"])
            if given is not None and not is_output:
                host[name] = np.ascontiguousarray(np.asarray(given, dtype=np.float32).reshape(arg["shape"]))
            else:
                host[name] = array_for(arg if not is_output else {**arg, "output": True})
            device[name] = session.upload(host[name])
        ptrs = {name: d.ptr for name, d in device.items()}
        session.ctx.timing_reset()
        times = []
        for rep in range(warmup + iters):
            session.ctx.timing(rep >= warmup)
            for spec in self.specs:
                for name in spec.zero_outputs:
                    session.ctx.memset(ptrs[name], 0, device[name].nbytes, session.stream)
                spec.launch(session.ctx, ptrs, session.stream)
            if rep >= warmup:
                session.sync()
                total = 0.0
                for phase in set(PHASE_OF[s.kind] for s in self.specs):
                    ms, _ = session.ctx.timing_read(phase)
                    total += ms
                session.ctx.timing_reset()
                times.append(total * 1e3)
        session.ctx.timing(False)
        session.sync()
        outputs, arrays, remaining = {}, {}, max_return
        for kernel in self.meta["kernels"]:
            for arg in kernel["args"]:
                if arg.get("output") and arg["name"] in self.meta.get("graph_outputs", [arg["name"]]):
                    arrays[arg["name"]] = session.download(device[arg["name"]])
                    outputs[arg["name"]] = output_summary(arrays[arg["name"]], arg, remaining)
                    remaining -= min(arrays[arg["name"]].size, remaining)
        for d in device.values():
            d.free()
        return {"ok": True, "median_us": statistics.median(times) if times else None, "iters": iters,
                "outputs": outputs, "kernels": [s.kind for s in self.specs],
                "timing_method": "CUDA events around each launch's kernels (b2k_timing), excludes resets and copies"}, arrays


def run(folder, device: int = 0, **kwargs) -> dict:
    """One launch request: recognise, allocate, run, summarise."""
    pipeline = Pipeline(folder)
    with api.Session(device) as session:
        result, _ = pipeline.run(session, **kwargs)
    return result
