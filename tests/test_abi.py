"""The C ABI: the built library loads and exports every symbol that
include/b200k.h declares (no compute calls: these run without a GPU)."""
from __future__ import annotations

import ctypes
import re
import subprocess

import pytest

from conftest import ROOT, pkg

HEADER = ROOT / "include" / "b200k.h"


def declared_functions() -> list[str]:
    text = re.sub(r"/\*.*?\*/", "", HEADER.read_text(), flags=re.S)
    return sorted(set(re.findall(r"\b(b2k_\w+)\s*\(", text)))


def test_header_declares_entry_points():
    names = declared_functions()
    for required in ("b2k_init", "b2k_gemm_tf32x3", "b2k_row_softmax_f32", "b2k_pointwise_f32"):
        assert required in names


def test_library_exports_every_declared_symbol():
    runtime = pkg("runtime")
    if not runtime.LIBRARY_PATH.exists():
        pkg("build").build()
    lib = ctypes.CDLL(str(runtime.LIBRARY_PATH))
    missing = [name for name in declared_functions() if not hasattr(lib, name)]
    assert not missing, missing
    out = subprocess.run(["nm", "-D", "--defined-only", str(runtime.LIBRARY_PATH)], capture_output=True, text=True)
    exported = set(re.findall(r"\bT (b2k_\w+)", out.stdout))
    assert set(declared_functions()) <= exported


def test_runtime_binds_every_declared_symbol():
    runtime = pkg("runtime")
    assert set(declared_functions()) <= set(runtime.exported_symbols())


def test_version_without_gpu():
    runtime = pkg("runtime")
    assert runtime.library().b2k_version() == 100


def test_bound_call_converts_once_and_checks_status():
    """BoundCall against a C function with the library's calling pattern
    (libc abs: the status is the return value)."""
    import ctypes as C
    import ctypes.util

    rt = pkg("runtime")
    libc = C.CDLL(ctypes.util.find_library("c"))
    libc.abs.argtypes, libc.abs.restype = [C.c_int], C.c_int
    seen = []

    class FakeCtx:
        lib = libc

        def check(self, status, call):
            seen.append((status, call))
            raise rt.B2KError(status, "failed", call)

    ok = rt.BoundCall(FakeCtx(), "abs", (0,))
    ok()
    ok()
    assert seen == []
    bad = rt.BoundCall(FakeCtx(), "abs", (-7,))
    with pytest.raises(rt.B2KError):
        bad()
    assert seen == [(7, "abs")]
