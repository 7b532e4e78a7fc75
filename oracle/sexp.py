"""CPU model of the selective subnormal-preserving exponential (test oracle).

Reference method (compile.py:2953-2965; docs/selective-exponential.md:15-36):

    t = f32(x * f32(log2 e))
    if t < -125:  r = ex2_ftz(t + 126) * 2^-126    (final multiply not flushed)
    else:         r = ex2_ftz(t)

``ex2_ftz`` is the hardware ``ex2.approx.ftz.f32``; the model evaluates it
exactly in float64 and rounds once, so it bounds rather than reproduces the
hardware's last bits.
"""
from __future__ import annotations

import numpy as np

LOG2E_F32 = np.float32(1.4426950408889634)
TWO_M126 = np.float64(2.0) ** -126
SUBNORMAL_ULP = np.float64(2.0) ** -149


def model(x) -> np.ndarray:
    x = np.asarray(x, dtype=np.float32)
    with np.errstate(over="ignore", invalid="ignore", under="ignore"):
        t = (x * LOG2E_F32).astype(np.float32)
        tiny = t < np.float32(-125.0)
        t2 = np.where(tiny, (t + np.float32(126.0)).astype(np.float32), t)
        r = np.exp2(t2.astype(np.float64))
        r = np.where(r < TWO_M126, 0.0, r).astype(np.float32)  # ftz output of ex2
        r = np.where(tiny, (r.astype(np.float64) * TWO_M126).astype(np.float32), r)
    return r.astype(np.float32)


def error_bound(x) -> np.ndarray:
    """Absolute error bound against float64 exp: the FP32 rounding of the
    argument product (|x| * 2^-24 relative, times ln 2 ... rounded up), two
    ulp of ex2.approx, and one subnormal quantum for the final rounding."""
    x = np.asarray(x, dtype=np.float64)
    exact = np.exp(x)
    rel = np.abs(x) * 2.0 ** -24 * 1.5 + 2.0 ** -21
    return exact * rel + SUBNORMAL_ULP


def check_against_exp(x, got) -> dict:
    x = np.asarray(x, dtype=np.float32)
    got = np.asarray(got, dtype=np.float32).astype(np.float64)
    exact = np.exp(x.astype(np.float64))
    err = np.abs(got - exact)
    bound = error_bound(x)
    finite = np.isfinite(exact) & (exact < 3.0e38)
    bad = finite & ~(err <= bound)
    return {"ok": bool(not bad.any()), "violations": int(bad.sum()),
            "max_abs_err": float(err[finite].max()) if finite.any() else 0.0,
            "worst_x": float(x[bad][0]) if bad.any() else None}
