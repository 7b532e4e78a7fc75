"""The reference's own GPU arithmetic for one 3xTF32 atom, run on the B200.

``tests/golden/tf32/synthetic_mma.ptx`` is the PTX text the reference's
``tf32_emitter.synthetic_ptx`` (tf32_emitter.py:120-222) emits for one
16 x 8 x 8 atom: one warp, ``cvt.rna.tf32.f32`` splits and three
``mma.sync.m16n8k8`` products combined as (hh + hl) + lh.  It was written by
``tests/golden/make_reference_ptx.py`` from the atom operands of
``tf32/vectors.npz``; this test JIT-loads it through the CUDA driver API
(``cuModuleLoadData``), launches it on those operands, and compares

* its output with the reference's CPU model of the same atom
  (``vectors.npz`` ``atom_c``, ``tf32_emitter.simulate``, tf32_emitter.py:43-61),
* this backend's tcgen05 3xTF32 GEMM (``b2k_gemm_tf32x3``, M = 16, N = 8,
  K = 8) with both,

at the model's normwise bound of 2e-6.  The PTX is loaded and run, never
inspected.
"""
from __future__ import annotations

import ctypes
import hashlib
import json

import numpy as np
import pytest

from conftest import GOLDEN
from oracle import tf32

pytestmark = pytest.mark.gpu

MODEL_BOUND = 2e-6


class Driver:
    """The few CUDA driver entry points needed to JIT-load and launch PTX."""

    def __init__(self):
        self.lib = ctypes.CDLL("libcuda.so.1")
        P, U = ctypes.c_void_p, ctypes.c_uint
        self.lib.cuModuleLoadData.argtypes = [ctypes.POINTER(P), ctypes.c_char_p]
        self.lib.cuModuleGetFunction.argtypes = [ctypes.POINTER(P), P, ctypes.c_char_p]
        self.lib.cuLaunchKernel.argtypes = [P, U, U, U, U, U, U, U, P, ctypes.POINTER(P), ctypes.POINTER(P)]
        self.lib.cuCtxSynchronize.argtypes = []
        self.lib.cuModuleUnload.argtypes = [P]
        self.lib.cuGetErrorString.argtypes = [ctypes.c_int, ctypes.POINTER(ctypes.c_char_p)]

    def check(self, status: int, what: str) -> None:
        if status != 0:
            msg = ctypes.c_char_p()
            self.lib.cuGetErrorString(status, ctypes.byref(msg))
            raise RuntimeError(f"{what}: CUDA driver error {status} ({(msg.value or b'').decode()})")

    def run_atom(self, ptx: bytes, entry: str, a_ptr: int, b_ptr: int, c_ptr: int) -> None:
        module, fn = ctypes.c_void_p(), ctypes.c_void_p()
        self.check(self.lib.cuModuleLoadData(ctypes.byref(module), ptx), "cuModuleLoadData")
        try:
            self.check(self.lib.cuModuleGetFunction(ctypes.byref(fn), module, entry.encode()), "cuModuleGetFunction")
            values = [ctypes.c_uint64(a_ptr), ctypes.c_uint64(b_ptr), ctypes.c_uint64(c_ptr)]
            params = (ctypes.c_void_p * 3)(*[ctypes.cast(ctypes.pointer(v), ctypes.c_void_p) for v in values])
            # one CTA of one warp, the launch the emitter documents
            self.check(self.lib.cuLaunchKernel(fn, 1, 1, 1, 32, 1, 1, 0, None, params, None), "cuLaunchKernel")
            self.check(self.lib.cuCtxSynchronize(), "cuCtxSynchronize")
        finally:
            self.lib.cuModuleUnload(module)


def reference_ptx() -> tuple[bytes, str]:
    record = json.loads((GOLDEN / "manifest.json").read_text())["reference_ptx"]
    data = (GOLDEN / record["file"]).read_bytes()
    assert hashlib.sha256(data).hexdigest() == record["sha256"], "fixture differs from the manifest"
    return data + b"\0", record["entry"]


def test_reference_atom_ptx_and_tcgen05_gemm_agree(ctx, torch_cuda):
    torch = torch_cuda
    vec = np.load(GOLDEN / "tf32" / "vectors.npz")
    a, b, model = vec["atom_a"], vec["atom_b"], vec["atom_c"]
    da, db = torch.from_numpy(a).cuda(), torch.from_numpy(b).cuda()
    ref_c = torch.full((16, 8), float("nan"), device="cuda")
    torch.cuda.synchronize()  # the primary context is current on this thread
    ptx, entry = reference_ptx()
    Driver().run_atom(ptx, entry, da.data_ptr(), db.data_ptr(), ref_c.data_ptr())
    ref_gpu = ref_c.cpu().numpy()
    ours_c = torch.full((16, 8), float("nan"), device="cuda")
    ctx.gemm(da.data_ptr(), db.data_ptr(), ours_c.data_ptr(), 16, 8, 8)
    ctx.sync()
    ours = ours_c.cpu().numpy()
    exact = a.astype(np.float64) @ b.astype(np.float64)
    assert np.isfinite(ref_gpu).all() and np.isfinite(ours).all()
    # the reference's GPU kernel against its own CPU model of the instruction
    assert tf32.normwise_error(ref_gpu, model) <= MODEL_BOUND, (ref_gpu - model)
    # the tcgen05 GEMM against the reference's model and its GPU result
    assert tf32.normwise_error(ours, model) <= MODEL_BOUND
    assert tf32.normwise_error(ours, ref_gpu) <= MODEL_BOUND
    assert tf32.normwise_error(ours, exact) <= 1e-5
