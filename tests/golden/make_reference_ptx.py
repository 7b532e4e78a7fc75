#!/usr/bin/env python3
"""Write the reference's own one-atom 3xTF32 PTX kernel as a test fixture.

Run from the repository root with the reference checkout available read-only:

    python tests/golden/make_reference_ptx.py --reference /path/to/emmy-hackathon-2026

The reference's ``tf32_emitter.synthetic_ptx`` (tf32_emitter.py:120-222) emits
PTX text for one warp that loads a 16 x 8 A and an 8 x 8 B (row-major FP32),
splits every operand with ``cvt.rna.tf32.f32``, issues the three
``mma.sync.m16n8k8`` products hi*hi, hi*lo, lo*hi into separate FP32
fragments and stores C = (hh + hl) + lh.  Its kernel parameters are the three
device pointers A, B, C; the entry name is given here.  The module imports
without the reference's missing ``emmy`` dependency, so this script runs it
on the atom operands of ``tf32/vectors.npz`` and writes the text, unread, to
``tf32/synthetic_mma.ptx``; its SHA-256 goes into ``manifest.json``.

The GPU test ``tests/test_gpu_reference_ptx.py`` JIT-loads that file on the
B200 through the CUDA driver API and runs it: the reference's own GPU
arithmetic for one atom, beside this backend's tcgen05 GEMM on the same
operands.  The PTX is loaded and run, never inspected.
"""
from __future__ import annotations

import argparse
import hashlib
import importlib.util
import json
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
ENTRY = "synthetic_mma"


def main() -> int:
    parser = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    parser.add_argument("--reference", type=Path, required=True)
    args = parser.parse_args()
    reference = args.reference.resolve()
    spec = importlib.util.spec_from_file_location("ref_tf32_emitter", reference / "tf32_emitter.py")
    module = importlib.util.module_from_spec(spec)
    sys.modules[spec.name] = module
    spec.loader.exec_module(module)
    vectors = np.load(HERE / "tf32" / "vectors.npz")
    text = module.synthetic_ptx(vectors["atom_a"], vectors["atom_b"], entry=ENTRY)
    out = HERE / "tf32" / "synthetic_mma.ptx"
    out.write_text(text)
    manifest_path = HERE / "manifest.json"
    manifest = json.loads(manifest_path.read_text())
    manifest["reference_ptx"] = {
        "file": "tf32/synthetic_mma.ptx", "sha256": hashlib.sha256(out.read_bytes()).hexdigest(), "entry": ENTRY,
        "params": ["A (u64, [16][8] f32)", "B (u64, [8][8] f32)", "C (u64, [16][8] f32)"], "launch": "1 CTA x 32",
        "source": "tf32_emitter.py:120-222 synthetic_ptx, run on tf32/vectors.npz atom_a / atom_b"}
    manifest_path.write_text(json.dumps(manifest, indent=1) + "\n")
    print(f"wrote {out.relative_to(HERE)} ({out.stat().st_size} bytes)")
    return 0


if __name__ == "__main__":
    sys.exit(main())
