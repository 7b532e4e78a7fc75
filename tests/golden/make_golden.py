#!/usr/bin/env python3
"""Regenerate the committed golden fixtures from a local checkout of the reference.

Run from the repository root, with the reference checkout available read-only:

    python tests/golden/make_golden.py --reference /path/to/emmy-hackathon-2026

Two kinds of fixture are written under ``tests/golden/``:

* ``cases/<name>-<id12>/`` -- byte-exact copies of the reference's bundled GPU
  regression cases (``tests/gpu-cases/cases/*`` and ``tests/variants/*``): the
  typed ``*.ir.json``, ``meta.json`` and ``case.json`` of every case, plus the
  ``inputs.npz`` / ``expected.npz`` payloads of every case whose arguments are
  all FP32 (the dtype of the hot path).  The expected outputs were produced by
  the reference's independent float64 NumPy equations and are the parity pins
  for the pointwise, reduction, softmax, matmul and attention families.
* ``tf32/vectors.npz`` -- outputs of the reference's own 3xTF32 CPU model
  (``tf32_emitter.tf32_rna``, ``simulate`` and ``simulate_matmul``,
  tf32_emitter.py:22-96) on seeded inputs and on edge values, produced by
  importing that module from the reference checkout.  These pin the oracle's
  vectorised restatement of the TF32 split and three-term accumulation.

The reference is never read at test time: the tests only read what this script
wrote, and ``manifest.json`` records the SHA-256 of every file.
"""
from __future__ import annotations

import argparse
import hashlib
import importlib.util
import json
import shutil
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent


def sha(path: Path) -> str:
    return hashlib.sha256(path.read_bytes()).hexdigest()


def all_f32(meta: dict) -> bool:
    return all(a.get("dtype", "f32") == "f32" for k in meta["kernels"] for a in k["args"])


def copy_cases(reference: Path, out: Path) -> list[dict]:
    manifest = json.loads((reference / "tests/gpu-cases/manifest.json").read_text())
    sources = [(c["name"], c["family"], reference / "tests/gpu-cases" / c["path"]) for c in manifest["cases"]]
    for variant in sorted((reference / "tests/variants").iterdir()):
        if variant.is_dir():
            sources.append((variant.name, "variant", variant))
    rows = []
    for name, family, folder in sources:
        case = json.loads((folder / "case.json").read_text())
        meta = json.loads((folder / "meta.json").read_text())
        ident = str(case.get("id", folder.name))[:12] if family != "variant" else "variant"
        dest = out / f"{name}-{ident}"
        dest.mkdir(parents=True, exist_ok=True)
        payload = all_f32(meta)
        files = [p for p in sorted(folder.iterdir())
                 if p.suffix == ".json" or (payload and p.suffix == ".npz")]
        for p in files:
            shutil.copyfile(p, dest / p.name)
        rows.append({"name": name, "family": family, "dir": dest.name,
                     "source": str(folder.relative_to(reference)),
                     "payload": payload, "rtol": meta.get("rtol"), "atol": meta.get("atol"),
                     "files": {p.name: sha(dest / p.name) for p in files}})
    return rows


def tf32_vectors(reference: Path, out: Path) -> dict:
    spec = importlib.util.spec_from_file_location("ref_tf32_emitter", reference / "tf32_emitter.py")
    module = importlib.util.module_from_spec(spec)
    sys.modules[spec.name] = module
    spec.loader.exec_module(module)
    rng = np.random.default_rng(20260101)
    f32 = np.float32
    # Edge values for the rounding model: ties, carries into the exponent,
    # max-finite (rounds to inf), subnormals, signed zeros and non-finite.
    specials = np.array([0.0, -0.0, 1.0, -1.0, 3.4028235e38, -3.4028235e38, 1e-45, -1e-45,
                         1.1754944e-38, 1.0e-40, np.inf, -np.inf, np.nan], dtype=f32)
    tie_bits = np.array([0x3F801000, 0x3F803000, 0x3F800FFF, 0x3F801001, 0x3FFFF000,
                         0x7F7FF000, 0x00001000, 0x807FF000], dtype=np.uint32).view(f32)
    sample = np.concatenate([specials, tie_bits, rng.standard_normal(4096).astype(f32),
                             (rng.standard_normal(1024) * 1e30).astype(f32),
                             (rng.standard_normal(1024) * 1e-38).astype(f32)])
    rna = np.array([module.tf32_rna(v) for v in sample], dtype=f32)
    atom_a = rng.uniform(-1, 1, (16, 8)).astype(f32)
    atom_b = rng.uniform(-1, 1, (8, 8)).astype(f32)
    atom_c = module.simulate(atom_a, atom_b)[0]
    mm_a = rng.uniform(-1, 1, (48, 64)).astype(f32)
    mm_b = rng.uniform(-1, 1, (64, 40)).astype(f32)
    mm_c = module.simulate_matmul(mm_a, mm_b)
    wide_a = (rng.standard_normal((24, 136)) * 8).astype(f32)
    wide_b = (rng.standard_normal((136, 16)) * 8).astype(f32)
    wide_c = module.simulate_matmul(wide_a, wide_b)
    # The max-finite x zero witness: the model yields NaN (inf*0) because
    # tf32_rna(max-finite) rounds to inf; kept as a pinned property.
    witness_a = np.full((16, 8), 3.4028235e38, dtype=f32)
    witness_b = np.zeros((8, 8), dtype=f32)
    with np.errstate(invalid="ignore"):
        witness_c = module.simulate(witness_a, witness_b)[0]
    arrays = dict(rna_in=sample, rna_out=rna, atom_a=atom_a, atom_b=atom_b, atom_c=atom_c,
                  mm_a=mm_a, mm_b=mm_b, mm_c=mm_c, wide_a=wide_a, wide_b=wide_b, wide_c=wide_c,
                  witness_a=witness_a, witness_b=witness_b, witness_c=witness_c)
    out.mkdir(parents=True, exist_ok=True)
    np.savez_compressed(out / "vectors.npz", **arrays)
    return {"file": "vectors.npz", "sha256": sha(out / "vectors.npz"),
            "source": "tf32_emitter.py:22-96 (tf32_rna, simulate, simulate_matmul)"}


def main() -> int:
    parser = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    parser.add_argument("--reference", type=Path, required=True)
    args = parser.parse_args()
    reference = args.reference.resolve()
    if not (reference / "tf32_emitter.py").is_file():
        print("not a reference checkout: " + str(reference), file=sys.stderr)
        return 2
    cases = copy_cases(reference, HERE / "cases")
    tf32 = tf32_vectors(reference, HERE / "tf32")
    (HERE / "manifest.json").write_text(json.dumps({"cases": cases, "tf32": tf32}, indent=1) + "\n")
    print(f"{len(cases)} cases, {sum(c['payload'] for c in cases)} with payloads; tf32 vectors written")
    return 0


if __name__ == "__main__":
    sys.exit(main())
