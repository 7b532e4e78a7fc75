"""Vectorised restatement of the reference's 3xTF32 CPU model (test oracle).

Reference: tf32_emitter.py:22-29 (``tf32_rna``), :43-61 (``simulate``) and
:64-96 (``simulate_matmul``).  The reference evaluates ``tf32_rna`` one element
at a time through ``np.vectorize``; here the same bit rule runs on whole
arrays so that it finishes at bench-sized shapes.
"""
from __future__ import annotations

import numpy as np


def tf32_rna(x) -> np.ndarray:
    """``cvt.rna.tf32.f32`` bit model (tf32_emitter.py:22-29).

    Finite inputs: ``(bits + 0x1000) & 0xFFFFE000`` (round to nearest, ties
    away from zero, on the 10-bit TF32 mantissa).  Non-finite inputs pass
    through.  Max-finite rounds up to infinity exactly as in the reference.
    """
    x = np.ascontiguousarray(x, dtype=np.float32)
    bits = x.view(np.uint32)
    rounded = ((bits + np.uint32(0x1000)) & np.uint32(0xFFFFE000)).view(np.float32)
    return np.where(np.isfinite(x), rounded, x).astype(np.float32)


def split(x) -> tuple[np.ndarray, np.ndarray]:
    """hi = rna(x), lo = rna(x - hi) with the subtraction in FP32 (tf32_emitter.py:50-53)."""
    x = np.asarray(x, dtype=np.float32)
    hi = tf32_rna(x)
    with np.errstate(invalid="ignore", over="ignore"):
        lo = tf32_rna((x - hi).astype(np.float32))
    return hi, lo


def simulate(a, b) -> np.ndarray:
    """One 16x8x8 atom, three exact f64 products rounded to f32, ``(hh + hl) + lh``
    (tf32_emitter.py:43-61)."""
    a = np.asarray(a, dtype=np.float32)
    b = np.asarray(b, dtype=np.float32)
    if a.shape != (16, 8) or b.shape != (8, 8):
        raise ValueError("one atom expects A=(16,8), B=(8,8)")
    return simulate_matmul(a, b, atom_k=8)


def simulate_matmul(a, b, atom_k: int = 8) -> np.ndarray:
    """Three separate f32 accumulators fed one exact 8-product dot per step,
    combined as ``(c_hh + c_hl) + c_lh`` in FP32 (tf32_emitter.py:64-96)."""
    a = np.asarray(a, dtype=np.float32)
    b = np.asarray(b, dtype=np.float32)
    if a.ndim != 2 or b.ndim != 2 or a.shape[1] != b.shape[0]:
        raise ValueError("simulate_matmul expects compatible rank-two operands")
    if a.shape[1] % atom_k:
        raise ValueError("K must be a multiple of the TF32 atom K extent")
    ah, al = split(a)
    bh, bl = split(b)
    ah, al, bh, bl = (t.astype(np.float64) for t in (ah, al, bh, bl))
    shape = (a.shape[0], b.shape[1])
    c_hh = np.zeros(shape, dtype=np.float32)
    c_hl = np.zeros(shape, dtype=np.float32)
    c_lh = np.zeros(shape, dtype=np.float32)
    with np.errstate(invalid="ignore", over="ignore"):
        for kk in range(0, a.shape[1], atom_k):
            s = slice(kk, kk + atom_k)
            c_hh = (c_hh.astype(np.float64) + ah[:, s] @ bh[s]).astype(np.float32)
            c_hl = (c_hl.astype(np.float64) + ah[:, s] @ bl[s]).astype(np.float32)
            c_lh = (c_lh.astype(np.float64) + al[:, s] @ bh[s]).astype(np.float32)
        return ((c_hh + c_hl).astype(np.float32) + c_lh).astype(np.float32)


def gemm_3xtf32(a, b) -> np.ndarray:
    """The 3xTF32 product with one f64 accumulation over the whole K extent.

    This is the backend's arithmetic contract (hi*hi + hi*lo + lo*hi, the
    lo*lo term dropped) without the per-atom FP32 rounding of
    :func:`simulate_matmul`; used at shapes where the per-atom loop is too slow.
    """
    ah, al = split(a)
    bh, bl = split(b)
    ah, al, bh, bl = (t.astype(np.float64) for t in (ah, al, bh, bl))
    with np.errstate(invalid="ignore", over="ignore"):
        return (ah @ bh + ah @ bl + al @ bh).astype(np.float32)


def normwise_error(got, exact) -> float:
    """max|got - exact| / max|exact| (the north-star's normwise 3xTF32 bound)."""
    got = np.asarray(got, dtype=np.float64)
    exact = np.asarray(exact, dtype=np.float64)
    scale = float(np.max(np.abs(exact))) or 1.0
    return float(np.max(np.abs(got - exact))) / scale
