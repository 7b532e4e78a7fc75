"""Seeded synthetic inputs for the five benchmark configurations.

The reference measures on small published problems and seeded scaled cases
(tests/performance/generators/suite.py:284-310 draws inputs with
``numpy.random.default_rng(seed)``); the configurations benchmarked here are
larger and are described in prose, so their inputs are drawn the same way
with fixed seeds and the stated distributions:

* add        -- a, b ~ U[-1, 1], n = 2^24                       (seeds 1001, 1002)
* softmax    -- x ~ N(0, var 16), 4096 x 8192, 1 % of the entries
                (seeded choice) set to -100                      (seeds 2001, 2002)
* gemm       -- A, B ~ U[-1, 1], 4096^3, row-major              (seeds 1001, 1002)
* ragged     -- A 4097 x 777, B^T 1000 x 777 ~ N(0, 1),
                bias[1000] ~ U[-0.5, 0.5]                        (seeds 1001, 1002, 4001)
* attention  -- Q, K, V ~ N(0, 1), [64 = 4 batches x 16 heads, 2048, 128]
                                                                 (seeds 3001, 3002, 3003)
"""
from __future__ import annotations

import numpy as np

F32 = np.float32

CONFIGS = {
    "add": {"n": 1 << 24},
    "softmax": {"rows": 4096, "cols": 8192},
    "gemm": {"m": 4096, "n": 4096, "k": 4096},
    "ragged": {"m": 4097, "n": 1000, "k": 777},
    "attention": {"batch": 4, "heads": 16, "seq": 2048, "head_dim": 128},
}


def rng(seed: int) -> np.random.Generator:
    return np.random.default_rng(seed)


def add_inputs(n: int = 1 << 24) -> tuple[np.ndarray, np.ndarray]:
    return (rng(1001).uniform(-1, 1, n).astype(F32), rng(1002).uniform(-1, 1, n).astype(F32))


def softmax_input(rows: int = 4096, cols: int = 8192) -> np.ndarray:
    x = rng(2001).normal(0.0, 4.0, (rows, cols)).astype(F32)
    count = max(1, (rows * cols) // 100)
    picked = rng(2002).choice(rows * cols, size=count, replace=False)
    x.reshape(-1)[picked] = F32(-100.0)
    return x


def gemm_inputs(m: int = 4096, n: int = 4096, k: int = 4096) -> tuple[np.ndarray, np.ndarray]:
    return (rng(1001).uniform(-1, 1, (m, k)).astype(F32), rng(1002).uniform(-1, 1, (k, n)).astype(F32))


def ragged_inputs(m: int = 4097, n: int = 1000, k: int = 777) -> tuple[np.ndarray, np.ndarray, np.ndarray]:
    return (rng(1001).standard_normal((m, k)).astype(F32),
            rng(1002).standard_normal((n, k)).astype(F32),
            rng(4001).uniform(-0.5, 0.5, n).astype(F32))


def attention_inputs(bh: int = 64, seq: int = 2048, d: int = 128) -> tuple[np.ndarray, np.ndarray, np.ndarray]:
    return tuple(rng(s).standard_normal((bh, seq, d)).astype(F32) for s in (3001, 3002, 3003))


# Algorithmic work per run (bytes or flop), the roofline numerators.
def add_bytes(n: int = 1 << 24) -> int:
    return 3 * 4 * n


def softmax_bytes(rows: int = 4096, cols: int = 8192) -> int:
    return 2 * 4 * rows * cols


def gemm_flop(m: int, n: int, k: int) -> int:
    return 2 * m * n * k


def attention_flop(bh: int, seq: int, d: int) -> int:
    return 4 * bh * seq * seq * d
