"""The reference's float64 NumPy equations per kernel family (test oracle).

Restated from tools/research_cases.py:74-103 (``reference``) and
tests/performance/generators/suite.py:192-234 (``stable_softmax``,
``_reference``): every input is promoted to float64, the plain mathematical
formula is evaluated, and the result is cast once to float32 per output --
the same rule that produced the bundled ``expected.npz`` files.
"""
from __future__ import annotations

import math

import numpy as np


def _f64(x) -> np.ndarray:
    return np.asarray(x, dtype=np.float32).astype(np.float64)


def pointwise(op: str, *args) -> np.ndarray:
    """research_cases.py:80-89 and suite.py:203-214."""
    xs = [_f64(a) for a in args]
    if op == "add":
        value = xs[0] + xs[1]
    elif op == "subtract":
        value = xs[0] - xs[1]
    elif op == "multiply":
        value = xs[0] * xs[1]
    elif op == "relu_mul":
        value = np.maximum(xs[0], 0.0) * xs[1]
    elif op == "scale_shift":
        value = xs[0] * xs[1].reshape(-1)[0] + xs[2].reshape(-1)[0]
    else:
        raise ValueError(f"unknown pointwise operation {op!r}")
    return value.astype(np.float32)


def stable_softmax(x, axis: int = -1) -> np.ndarray:
    """suite.py:192-196: subtract the row max, exp, normalise (float64)."""
    z = _f64(x)
    z = z - np.max(z, axis=axis, keepdims=True)
    e = np.exp(z)
    return e / np.sum(e, axis=axis, keepdims=True)


def softmax(x) -> np.ndarray:
    return stable_softmax(x).astype(np.float32)


def matmul(a, b) -> np.ndarray:
    """research_cases.py:92 / suite.py:219-221: ``x @ y`` in float64."""
    return (_f64(a) @ _f64(b)).astype(np.float32)


def matmul_bias_relu(a, b_t, bias) -> np.ndarray:
    """The ragged fused-epilogue GEMM: relu(A @ B^T + bias) in float64 (B stored N x K)."""
    value = _f64(a) @ _f64(b_t).T + _f64(bias)[None, :]
    return np.maximum(value, 0.0).astype(np.float32)


def attention(q, kt, v, scale) -> np.ndarray:
    """research_cases.py:95-98 / suite.py:230-233:
    softmax((q @ kt) / scale) @ v, float64, for one head (q: S x D, kt: D x S)."""
    scores = (_f64(q) @ _f64(kt)) / float(scale)
    return (stable_softmax(scores) @ _f64(v)).astype(np.float32)


def attention_batched(q, k, v, scale: float | None = None, heads_per_pass: int = 8) -> np.ndarray:
    """Per-(batch, head) :func:`attention` with K stored like Q (``[BH, S, D]``),
    evaluated a few heads at a time (batched float64 BLAS matmuls) so that the
    float64 score tensor stays a few hundred MB at S = 2048."""
    q = np.asarray(q, dtype=np.float32)
    scale = math.sqrt(q.shape[-1]) if scale is None else scale
    out = np.empty(q.shape[:-1] + (np.shape(v)[-1],), dtype=np.float32)
    for h in range(0, q.shape[0], heads_per_pass):
        qh, kh, vh = _f64(q[h:h + heads_per_pass]), _f64(k[h:h + heads_per_pass]), _f64(v[h:h + heads_per_pass])
        scores = np.matmul(qh, np.swapaxes(kh, 1, 2)) / float(scale)
        out[h:h + heads_per_pass] = np.matmul(stable_softmax(scores), vh).astype(np.float32)
    return out


def rmsnorm(x, w=None, eps: float = 1e-5) -> np.ndarray:
    """suite.py:222-225 (with weight) / research_cases.py:99-100 (without)."""
    x = _f64(x)
    value = x / np.sqrt(np.mean(x * x, axis=-1, keepdims=True) + eps)
    if w is not None:
        value = value * _f64(w)
    return value.astype(np.float32)


def l2norm(x, eps: float = 0.0) -> np.ndarray:
    """suite.py:226-229 (eps 0) / research_cases.py:101-102."""
    x = _f64(x)
    return (x / np.sqrt(np.sum(x * x, axis=-1, keepdims=True) + eps)).astype(np.float32)


def mean(x) -> np.ndarray:
    """r03_mean: the float64 mean of all elements."""
    return np.asarray([_f64(x).mean()], dtype=np.float32)


def array_sum(x) -> np.ndarray:
    """suite.py:215-216 (``reduction``)."""
    return np.asarray([_f64(x).sum()], dtype=np.float32)


def row_sum(x) -> np.ndarray:
    """suite.py:217-218 (``row_sum``)."""
    return _f64(x).sum(axis=1).astype(np.float32)


def allclose_report(got, expected, rtol: float, atol: float) -> tuple[bool, int, float]:
    """The reference's comparison rule (tools/research_gpu.py:71-86):
    elementwise ``np.isclose(got, expected, rtol, atol)``; returns
    (all close, mismatch count, max abs error)."""
    got = np.asarray(got)
    expected = np.asarray(expected)
    if got.shape != expected.shape:
        return False, got.size, float("inf")
    close = np.isclose(got, expected, rtol=rtol, atol=atol, equal_nan=False)
    diff = np.abs(got.astype(np.float64) - expected.astype(np.float64))
    finite = diff[np.isfinite(diff)]
    return bool(close.all()), int((~close).sum()), float(finite.max()) if finite.size else 0.0
