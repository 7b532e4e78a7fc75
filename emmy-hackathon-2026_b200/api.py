"""Public Python API over the C ABI, for callers that bring host arrays.

:class:`Session` owns one library context, device buffers allocated through
the library (no PyTorch), page-locked host staging buffers, and the host <->
device copies around each kernel -- the work the reference's runner does per
launch request (tools/local_runner.py:246-342: allocate, copy in, reset
``zero_outputs``, launch, copy out).
"""
from __future__ import annotations

import ctypes as C
import math

import numpy as np

from . import runtime

F32 = np.dtype(np.float32)


class DeviceArray:
    """A device allocation made by the library (freed on :meth:`free`)."""

    def __init__(self, session: "Session", shape: tuple[int, ...], dtype=F32):
        self.session, self.shape, self.dtype = session, tuple(int(s) for s in shape), np.dtype(dtype)
        self.nbytes = int(math.prod(self.shape)) * self.dtype.itemsize
        self.ptr = session.ctx.malloc(max(1, self.nbytes))

    @property
    def size(self) -> int:
        return int(math.prod(self.shape))

    def free(self) -> None:
        if self.ptr:
            self.session.ctx.free(self.ptr)
            self.ptr = 0


class Session:
    """One device, one context, one stream (the legacy default stream unless given)."""

    def __init__(self, device: int = 0, stream: int = 0):
        self.ctx = runtime.Context(device)
        self.stream = stream
        self._pinned: list[int] = []

    def close(self) -> None:
        for ptr in self._pinned:
            self.ctx.host_free(ptr)
        self._pinned.clear()
        self.ctx.close()

    def __enter__(self) -> "Session":
        return self

    def __exit__(self, *exc) -> None:
        self.close()

    # --- memory --------------------------------------------------------------
    def empty(self, shape, dtype=F32) -> DeviceArray:
        return DeviceArray(self, tuple(shape), dtype)

    def pinned(self, shape, dtype=F32) -> np.ndarray:
        """A NumPy array backed by page-locked host memory (lives with the session)."""
        dtype = np.dtype(dtype)
        count = int(math.prod(shape))
        ptr = self.ctx.host_alloc(max(1, count * dtype.itemsize))
        self._pinned.append(ptr)
        raw = (C.c_uint8 * max(1, count * dtype.itemsize)).from_address(ptr)
        return np.frombuffer(raw, dtype=dtype, count=count).reshape(shape)

    def upload(self, host: np.ndarray, out: DeviceArray | None = None) -> DeviceArray:
        host = np.ascontiguousarray(host)
        out = out or self.empty(host.shape, host.dtype)
        if out.nbytes != host.nbytes:
            raise ValueError("upload: size mismatch")
        if host.nbytes:
            self.ctx.htod(out.ptr, host.ctypes.data, host.nbytes, self.stream)
        return out

    def download(self, dev: DeviceArray, out: np.ndarray | None = None) -> np.ndarray:
        out = np.empty(dev.shape, dev.dtype) if out is None else out
        if not out.flags.c_contiguous or out.nbytes != dev.nbytes:
            raise ValueError("download: destination must be contiguous and the same size")
        if dev.nbytes:
            self.ctx.dtoh(out.ctypes.data, dev.ptr, dev.nbytes, self.stream)
        return out

    def sync(self) -> None:
        self.ctx.sync(self.stream)

    # --- kernels on device arrays ---------------------------------------------
    def gemm(self, a: DeviceArray, b: DeviceArray, c: DeviceArray, *, b_layout: str = "kn",
             bias: DeviceArray | None = None, relu: bool = False) -> None:
        m, k = a.shape
        n = b.shape[1] if b_layout == "kn" else b.shape[0]
        if c.shape != (m, n):
            raise ValueError(f"gemm: output shape {c.shape} != {(m, n)}")
        self.ctx.gemm(a.ptr, b.ptr, c.ptr, m, n, k, b_layout=runtime.B_KN if b_layout == "kn" else runtime.B_NK,
                      bias=bias.ptr if bias is not None else 0, relu=relu, stream=self.stream)

    def row_softmax(self, x: DeviceArray, y: DeviceArray) -> None:
        rows, cols = x.shape
        self.ctx.row_softmax(x.ptr, y.ptr, rows, cols, stream=self.stream)

    def pointwise(self, program, inputs: list[DeviceArray], out: DeviceArray) -> None:
        self.ctx.pointwise(program, [t.ptr for t in inputs], out.ptr, out.size, stream=self.stream)

    # --- end to end from host arrays --------------------------------------------
    # One library call per operation: the inputs are copied in slab by slab on
    # a copy stream, each slab computes as soon as it has landed, and finished
    # output slabs are copied out on a second copy stream (b2k_*_host).  The
    # calls are asynchronous: `out` is complete after :meth:`sync`.  Host
    # arrays from :meth:`pinned` give full copy/compute overlap.
    @staticmethod
    def _host_in(x: np.ndarray) -> np.ndarray:
        x = np.asarray(x)
        if x.dtype != F32 or not x.flags.c_contiguous:
            raise ValueError("host inputs must be C-contiguous float32 arrays")
        return x

    @staticmethod
    def _host_out(out: np.ndarray | None, shape: tuple) -> np.ndarray:
        if out is None:
            return np.empty(shape, F32)
        if out.dtype != F32 or not out.flags.c_contiguous or out.shape != tuple(shape):
            raise ValueError(f"output must be a C-contiguous float32 array of shape {tuple(shape)}")
        return out

    def gemm_host(self, a: np.ndarray, b: np.ndarray, out: np.ndarray | None = None, *, b_layout: str = "kn",
                  bias: np.ndarray | None = None, relu: bool = False) -> np.ndarray:
        a, b = self._host_in(a), self._host_in(b)
        m, k = a.shape
        n = b.shape[1] if b_layout == "kn" else b.shape[0]
        out = self._host_out(out, (m, n))
        bias = self._host_in(bias) if bias is not None else None
        self.ctx.gemm_host(a.ctypes.data, b.ctypes.data, out.ctypes.data, m, n, k,
                           b_layout=runtime.B_KN if b_layout == "kn" else runtime.B_NK,
                           bias=bias.ctypes.data if bias is not None else 0, relu=relu, stream=self.stream)
        return out

    def row_softmax_host(self, x: np.ndarray, out: np.ndarray | None = None) -> np.ndarray:
        x = self._host_in(x)
        rows, cols = x.shape
        out = self._host_out(out, x.shape)
        self.ctx.row_softmax_host(x.ctypes.data, out.ctypes.data, rows, cols, stream=self.stream)
        return out

    def pointwise_host(self, program, inputs: list[np.ndarray], out: np.ndarray) -> np.ndarray:
        inputs = [self._host_in(t) for t in inputs]
        out = self._host_out(out, out.shape)
        self.ctx.pointwise_host(program, [t.ctypes.data for t in inputs], out.ctypes.data, out.size,
                                stream=self.stream)
        return out

    def attention_host(self, q: np.ndarray, k: np.ndarray, v: np.ndarray, out: np.ndarray | None = None, *,
                       scale: float | None = None, k_layout: str = "sd") -> np.ndarray:
        """q [bh, s_q, d], k [bh, s_kv, d] (or [bh, d, s_kv] with k_layout "ds"), v [bh, s_kv, dv]."""
        q, k, v = self._host_in(q), self._host_in(k), self._host_in(v)
        bh, s_q, d = q.shape
        s_kv, dv = v.shape[1], v.shape[2]
        out = self._host_out(out, (bh, s_q, dv))
        self.ctx.attention_host(q.ctypes.data, k.ctypes.data, v.ctypes.data, out.ctypes.data, bh, s_q, s_kv, d, dv,
                                scale=scale, k_layout=runtime.K_SD if k_layout == "sd" else runtime.K_DS,
                                stream=self.stream)
        return out
