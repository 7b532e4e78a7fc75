"""Build ``libb200k.so`` (the C-ABI kernel library) in-tree with nvcc for sm_100a.

Each ``csrc/*.cu`` file is compiled to an object under ``_build/`` (rebuilt
when it or a header is newer than its object) and linked into
``libb200k.so`` beside this file, so the library travels with the source tree.
"""
from __future__ import annotations

import os
import shutil
import subprocess
import sys
from concurrent.futures import ThreadPoolExecutor
from pathlib import Path

PACKAGE = Path(__file__).resolve().parent
REPO = PACKAGE.parent
CSRC = PACKAGE / "csrc"
INCLUDE = REPO / "include"
BUILD = REPO / "_build" / "b200k"
LIBRARY = PACKAGE / "libb200k.so"

ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]
CFLAGS = ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC", "-Xptxas", "-v",
          "--expt-relaxed-constexpr", "-DNDEBUG"]


def nvcc() -> str:
    found = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not Path(found).exists():
        raise RuntimeError("nvcc not found: the CUDA toolkit is required to build libb200k.so")
    return found


def sources() -> list[Path]:
    return sorted(CSRC.glob("*.cu"))


def headers() -> list[Path]:
    return sorted(CSRC.glob("*.cuh")) + sorted(INCLUDE.glob("*.h"))


def _compile(src: Path, verbose: bool) -> tuple[Path, str]:
    obj = BUILD / (src.stem + ".o")
    newest_dep = max([src.stat().st_mtime] + [h.stat().st_mtime for h in headers()])
    if obj.exists() and obj.stat().st_mtime >= newest_dep:
        return obj, ""
    cmd = [nvcc(), *ARCH_FLAGS, *CFLAGS, f"-I{INCLUDE}", f"-I{CSRC}", "-c", str(src), "-o", str(obj)]
    done = subprocess.run(cmd, capture_output=True, text=True)
    if done.returncode:
        raise RuntimeError(f"nvcc failed for {src.name}:\n{done.stderr[-6000:]}")
    log = BUILD / (src.stem + ".ptxas.txt")
    log.write_text(done.stderr)
    if verbose:
        print(done.stderr, file=sys.stderr)
    return obj, done.stderr


def build(verbose: bool = False) -> Path:
    """Compile and link ``libb200k.so``; returns its path."""
    BUILD.mkdir(parents=True, exist_ok=True)
    srcs = sources()
    with ThreadPoolExecutor(max_workers=min(8, len(srcs))) as pool:
        objs = [obj for obj, _ in pool.map(lambda s: _compile(s, verbose), srcs)]
    if LIBRARY.exists() and LIBRARY.stat().st_mtime >= max(o.stat().st_mtime for o in objs):
        return LIBRARY
    tmp = LIBRARY.with_suffix(".so.tmp")
    cmd = [nvcc(), *ARCH_FLAGS, "-shared", "-o", str(tmp), *map(str, objs)]
    done = subprocess.run(cmd, capture_output=True, text=True)
    if done.returncode:
        raise RuntimeError(f"nvcc link failed:\n{done.stderr[-4000:]}")
    os.replace(tmp, LIBRARY)
    return LIBRARY


if __name__ == "__main__":
    print(build(verbose="-v" in sys.argv))
