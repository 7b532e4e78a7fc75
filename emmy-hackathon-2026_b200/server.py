"""Loopback HTTP runner over this back end: ``/health``, ``/compile``, ``/run``.

The reference serves the same three paths on a loopback-only port
(tools/local_runner.py:345-375).  Its ``/compile`` assembles PTX into a cached
cubin and returns the cubin's content hash (:178-218); its ``/run`` launches a
compiled kernel in a fresh worker process, one launch at a time, with a time
limit on the worker (:220-246).  Here the unit that is compiled is the Kernel
IR itself:

* ``POST /compile`` ``{"meta": <meta.json>, "ir": <graph>}`` (or ``"irs":
  {entry: <graph>}`` for a multi-kernel pipeline) recognises every metadata
  kernel through ``frontend.compile_path``, caches the files under the SHA-256
  of their canonical JSON and replies ``{"ok": true, "kernel_id": ...,
  "kernels": [<KernelSpec.describe()>...]}``;
* ``POST /run`` ``{"kernel_id": ...}`` (or the ``/compile`` fields) plus
  optional ``inputs`` (``{name: {"data": [...]} | {"seed": n}}``), ``warmup``,
  ``iters`` and ``max_return`` runs the pipeline through the C ABI in a fresh
  worker process (``runner.Pipeline``: seeded or given inputs, ``zero_outputs``
  cleared before every launch, CUDA-event timing, output summaries).

Failures keep the reference's reply shape ``{"ok": false, "stage": ...,
"stderr": ...}``: HTTP 422 for an invalid request, 404 for an unknown path,
500 for an internal error, 200 with ``stage`` ``compile`` / ``lookup`` /
``busy`` / ``run`` otherwise.  The server binds 127.0.0.1 only.
"""
from __future__ import annotations

import argparse
import ctypes as C
import hashlib
import json
import math
import os
import re
import signal
import subprocess
import sys
import tempfile
import threading
from http.server import BaseHTTPRequestHandler, ThreadingHTTPServer
from pathlib import Path

from . import frontend, runner

MAX_BODY = 96 * 1024 * 1024     # tools/local_runner.py:34
MAX_ELEMENTS = 2 ** 26          # total buffer elements of one request (:32)
MAX_RETURN = 2 ** 22            # output values returned (:33)
WORKER_SECONDS = 60             # the worker creates a context, loads the library, runs, copies out
PACKAGE_ROOT = Path(__file__).resolve().parent
ENTRY_RE = re.compile(r"[A-Za-z_$][\w$]*")
KERNEL_ID_RE = re.compile(r"[a-f0-9]{64}")


class Invalid(ValueError):
    """A malformed request (HTTP 422)."""


def _integer(value, name, lower, upper) -> int:
    if type(value) is not int or not lower <= value <= upper:
        raise Invalid(f"{name} must be an integer in [{lower}, {upper}]")
    return value


def _pipeline_files(body) -> dict:
    """{file name: JSON object} of one pipeline request (meta + IR graphs)."""
    if not isinstance(body, dict):
        raise Invalid("request must be an object")
    meta = body.get("meta")
    if not isinstance(meta, dict) or not isinstance(meta.get("kernels"), list) or not meta["kernels"]:
        raise Invalid("meta must be a meta.json object with a non-empty kernels list")
    total = 0
    for kernel in meta["kernels"]:
        if not isinstance(kernel, dict) or not isinstance(kernel.get("entry"), str) \
                or not ENTRY_RE.fullmatch(kernel["entry"]):
            raise Invalid("each metadata kernel needs an identifier entry")
        for arg in kernel.get("args", []):
            shape = arg.get("shape") if isinstance(arg, dict) else None
            if not isinstance(shape, list) or len(shape) > 8:
                raise Invalid("each argument needs a shape of at most 8 dimensions")
            for dim in shape:
                _integer(dim, "shape dimension", 0, MAX_ELEMENTS)
            total += math.prod(shape)
    if total > MAX_ELEMENTS:
        raise Invalid("total buffer elements exceed 2^26")
    files = {"meta.json": meta}
    if "irs" in body:
        irs = body["irs"]
        if not isinstance(irs, dict) or not irs:
            raise Invalid("irs must map entry names to IR graphs")
        for entry, graph in irs.items():
            if not isinstance(entry, str) or not ENTRY_RE.fullmatch(entry) or not isinstance(graph, dict):
                raise Invalid("irs must map entry names to IR graphs")
            files[f"{entry}.ir.json"] = graph
    elif isinstance(body.get("ir"), dict):
        files[f"{meta['kernels'][0]['entry']}.ir.json"] = body["ir"]
    else:
        raise Invalid("give ir (one graph) or irs (entry -> graph)")
    return files


def _run_options(body) -> dict:
    options = {"warmup": _integer(body.get("warmup", 5), "warmup", 0, 20),
               "iters": _integer(body.get("iters", 20), "iters", 1, 200),
               "max_return": _integer(body.get("max_return", 4096), "max_return", 0, MAX_RETURN)}
    inputs = body.get("inputs", {})
    if not isinstance(inputs, dict):
        raise Invalid("inputs must map argument names to {data} or {seed}")
    for name, given in inputs.items():
        if not isinstance(given, dict) or len(given) != 1 or not ({"data", "seed"} & given.keys()):
            raise Invalid(f"input {name!r} needs exactly one of data or seed")
        if "data" in given and not isinstance(given["data"], list):
            raise Invalid(f"input {name!r}: data must be a list")
        if "seed" in given:
            _integer(given["seed"], f"input {name!r} seed", 0, 2 ** 64 - 1)
    options["inputs"] = inputs
    return options


class Runner:
    """The server's state: a content-addressed pipeline cache and the run lock."""

    def __init__(self, cache, device: int = 0):
        self.cache = Path(cache)
        self.cache.mkdir(parents=True, exist_ok=True)
        self.device = device
        self.compile_lock = threading.Lock()
        self.run_lock = threading.Lock()

    def compile(self, body) -> dict:
        files = _pipeline_files(body)
        key = hashlib.sha256(json.dumps(files, sort_keys=True, ensure_ascii=True).encode()).hexdigest()
        folder = self.cache / key
        with self.compile_lock:
            record = folder / "compile.json"
            if record.exists():
                return json.loads(record.read_text())
            folder.mkdir(exist_ok=True)
            for name, value in files.items():
                (folder / name).write_text(json.dumps(value))
            try:
                pipeline = runner.Pipeline(folder)
            except (frontend.Unsupported, frontend.IRError, KeyError, TypeError) as exc:
                result = {"ok": False, "stage": "compile", "stderr": f"{type(exc).__name__}: {exc}"}
            else:
                result = {"ok": True, "kernel_id": key, "kernels": [s.describe() for s in pipeline.specs]}
            record.write_text(json.dumps(result))
            return result

    def run(self, body) -> dict:
        if not isinstance(body, dict):
            raise Invalid("request must be an object")
        options = _run_options(body)
        if "kernel_id" in body:
            if not isinstance(body["kernel_id"], str) or not KERNEL_ID_RE.fullmatch(body["kernel_id"]):
                raise Invalid("kernel_id must be a SHA256 hex digest")
            key = body["kernel_id"]
        else:
            compiled = self.compile(body)
            if not compiled["ok"]:
                return compiled
            key = compiled["kernel_id"]
        folder = self.cache / key
        record = folder / "compile.json"
        if not record.is_file() or not json.loads(record.read_text()).get("ok"):
            return {"ok": False, "stage": "lookup", "stderr": "unknown kernel_id"}
        if not self.run_lock.acquire(blocking=False):
            return {"ok": False, "stage": "busy", "stderr": "one launch already active"}
        try:
            with tempfile.TemporaryDirectory(prefix="run-", dir=self.cache) as tmp:
                request, result = Path(tmp) / "request.json", Path(tmp) / "result.json"
                request.write_text(json.dumps({**options, "folder": str(folder), "device": self.device,
                                               "parent_pid": os.getpid()}))
                env = dict(os.environ)
                env["PYTHONPATH"] = os.pathsep.join(filter(None, [str(PACKAGE_ROOT.parent), env.get("PYTHONPATH")]))
                try:
                    done = subprocess.run([sys.executable, "-m", f"{PACKAGE_ROOT.name}.server", "--worker",
                                           str(request), str(result)], cwd=str(PACKAGE_ROOT.parent), env=env,
                                          capture_output=True, text=True, timeout=WORKER_SECONDS)
                except subprocess.TimeoutExpired:
                    return {"ok": False, "stage": "run", "stderr": f"worker exceeded {WORKER_SECONDS} seconds"}
                if done.returncode or not result.is_file():
                    return {"ok": False, "stage": "run", "stderr": done.stderr[-4000:] or f"worker exit {done.returncode}"}
                return json.loads(result.read_text())
        finally:
            self.run_lock.release()


def worker(request: dict) -> dict:
    """One launch request in a fresh process that owns its CUDA context; any
    error ends the process (tools/local_runner.py:249-260, 336)."""
    if sys.platform.startswith("linux"):
        libc = C.CDLL(None, use_errno=True)
        libc.prctl.argtypes = [C.c_int, C.c_ulong, C.c_ulong, C.c_ulong, C.c_ulong]
        if libc.prctl(1, signal.SIGKILL, 0, 0, 0):       # PR_SET_PDEATHSIG: die with the server
            raise OSError(C.get_errno(), "cannot set the worker's parent-death signal")
        if os.getppid() != request["parent_pid"]:
            raise RuntimeError("the server exited before the worker started")
    pipeline = runner.Pipeline(request["folder"])
    inputs = {}
    for name, given in request["inputs"].items():
        arg = pipeline.args.get(name)
        if arg is None:
            raise ValueError(f"input {name!r} is not an argument of the pipeline")
        inputs[name] = runner.array_for({**arg, **given, "output": False})
    from . import api
    with api.Session(request["device"]) as session:
        result, _ = pipeline.run(session, inputs=inputs, warmup=request["warmup"], iters=request["iters"],
                                 max_return=request["max_return"])
    return result


def handler_for(state: Runner):
    class Handler(BaseHTTPRequestHandler):
        def log_message(self, fmt, *args):  # quiet: the replies carry the outcome
            pass

        def reply(self, status: int, body: dict) -> None:
            data = json.dumps(body).encode()
            self.send_response(status)
            self.send_header("Content-Type", "application/json")
            self.send_header("Content-Length", str(len(data)))
            self.end_headers()
            self.wfile.write(data)

        def do_GET(self):
            if self.path != "/health":
                return self.reply(404, {"ok": False, "stage": "request", "stderr": "unknown path"})
            library = (PACKAGE_ROOT / "libb200k.so").is_file()
            self.reply(200, {"ok": True, "can_compile": True, "can_run": library, "backend": "b200k sm_100a",
                             "device": state.device, "families": sorted({k for k, _ in frontend.FAMILIES}),
                             "implementation": "Kernel-IR runner over the b200k C ABI"})

        def do_POST(self):
            if self.path not in ("/compile", "/run"):
                return self.reply(404, {"ok": False, "stage": "request", "stderr": "unknown path"})
            try:
                length = _integer(int(self.headers.get("Content-Length", "0")), "body bytes", 1, MAX_BODY)
                self.connection.settimeout(10)
                body = json.loads(self.rfile.read(length))
                self.reply(200, state.compile(body) if self.path == "/compile" else state.run(body))
            except (Invalid, ValueError, TypeError, OverflowError) as exc:
                self.reply(422, {"ok": False, "stage": "request", "stderr": str(exc)})
            except Exception as exc:  # reply, keep serving
                self.reply(500, {"ok": False, "stage": "internal", "stderr": f"{type(exc).__name__}: {exc}"})
    return Handler


def serve(port: int = 0, cache=None, device: int = 0) -> ThreadingHTTPServer:
    """A server bound to 127.0.0.1 (``port`` 0 picks a free one); call
    ``serve_forever`` on it, ``shutdown`` from another thread to stop."""
    cache = cache or Path(tempfile.gettempdir()) / "b200k-runner"
    return ThreadingHTTPServer(("127.0.0.1", port), handler_for(Runner(cache, device)))


def main(argv=None) -> int:
    argv = sys.argv[1:] if argv is None else argv
    if len(argv) == 3 and argv[0] == "--worker":
        result = worker(json.loads(Path(argv[1]).read_text()))
        Path(argv[2]).write_text(json.dumps(result))
        return 0
    parser = argparse.ArgumentParser(description="loopback Kernel-IR runner over the b200k back end")
    parser.add_argument("--port", type=int, default=8000)
    parser.add_argument("--cache", default=None)
    parser.add_argument("--device", type=int, default=0)
    args = parser.parse_args(argv)
    server = serve(args.port, args.cache, args.device)
    print(f"serving on http://127.0.0.1:{server.server_address[1]}", flush=True)
    try:
        server.serve_forever()
    except KeyboardInterrupt:
        pass
    return 0


if __name__ == "__main__":
    sys.exit(main())
