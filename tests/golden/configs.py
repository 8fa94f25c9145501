"""Seeded synthetic inputs of the five benchmark configurations of the W8A8
bposit path (no dataset is involved; every input is drawn here).

Shared by the full-size parity tests, the generator of the committed C5
hashes (make_c5_golden.py) and bench.py, so that all three see the same
bits.  numpy's ``default_rng(seed)`` is the generator; float32 normals are
drawn with ``standard_normal(..., dtype=np.float32)`` in row-major order.

* C1  W8A8 linear 128 x 2048 x 11008: x ~ N(0, 1), w ~ N(0, 0.02), seed 0.
* C2  exact sums: see ``oracle.bposit_oracle.exact_sum_inputs``.
* C3  square int8 GEMMs: A, B uniform int8 in [-127, 127].
* C4  transformer shapes, per-token / per-channel: activations ~ N(0, 1)
      with 1% of the channels (input features) scaled by 20, weights
      ~ N(0, 0.02).
* C5  16384 x 8192 x 28672 W8A8: x ~ N(0, 1), w ~ N(0, 0.02), seed 0.

Weights are returned in ``nn.Linear`` layout ``[N, K]`` (= the column-major
``[K, N]`` of the C ABI); activations row-major ``[M, K]``.
"""
from __future__ import annotations

import numpy as np

C1 = (128, 2048, 11008)                 # M, K, N
C4_GATE = (2048, 4096, 14336)           # M, K, N
C4_QKT = (32, 2048, 2048, 128)          # heads, queries, keys, head dim
C4_FFN = (2048, 2048, 11008)            # tokens, hidden, intermediate
C5 = (16384, 8192, 28672)               # M, K, N


def normal(rng: np.random.Generator, shape, std: float = 1.0) -> np.ndarray:
    x = rng.standard_normal(shape, dtype=np.float32)
    if std != 1.0:
        x *= np.float32(std)
    return x


def with_outliers(rng: np.random.Generator, x: np.ndarray, frac: float = 0.01,
                  factor: float = 20.0) -> np.ndarray:
    """Scale ``frac`` of the last-axis channels (at least one) by ``factor``."""
    K = x.shape[-1]
    cols = rng.choice(K, max(1, int(K * frac)), replace=False)
    x[..., cols] *= np.float32(factor)
    return x


def c1_inputs(seed: int = 0):
    """(x [128, 2048], w [11008, 2048]) fp32."""
    M, K, N = C1
    rng = np.random.default_rng(seed)
    x = normal(rng, (M, K))
    w = normal(rng, (N, K), 0.02)
    return x, w


def c3_operands(M: int, N: int, K: int, seed: int = 0):
    """(A [M, K], B [N, K]) int8 uniform in [-127, 127]."""
    rng = np.random.default_rng(seed)
    A = rng.integers(-127, 128, (M, K), dtype=np.int8)
    B = rng.integers(-127, 128, (N, K), dtype=np.int8)
    return A, B


def c4_linear_inputs(M: int, K: int, N: int, seed: int = 0):
    """(x [M, K] with outlier channels, w [N, K] ~ N(0, 0.02))."""
    rng = np.random.default_rng(seed)
    x = with_outliers(rng, normal(rng, (M, K)))
    w = normal(rng, (N, K), 0.02)
    return x, w


def c4_qkt_inputs(seed: int = 0):
    """(q [heads, S, D], k [heads, S, D]) fp32, each with outlier channels."""
    H, S, T, D = C4_QKT
    rng = np.random.default_rng(seed)
    q = with_outliers(rng, normal(rng, (H, S, D)))
    k = with_outliers(rng, normal(rng, (H, T, D)))
    return q, k


def c4_ffn_inputs(seed: int = 0):
    """(x [M, D] with outlier channels, w_gate [F, D], w_up [F, D], w_down [D, F])."""
    M, D, F = C4_FFN
    rng = np.random.default_rng(seed)
    x = with_outliers(rng, normal(rng, (M, D)))
    wg = normal(rng, (F, D), 0.02)
    wu = normal(rng, (F, D), 0.02)
    wd = normal(rng, (D, F), 0.02)
    return x, wg, wu, wd


def c5_inputs(M: int = C5[0], seed: int = 0):
    """(x [M, 8192], w [28672, 8192]) fp32.  The weights are drawn first, so a
    run with fewer rows (M < 16384) sees the same weights and the first M
    rows of the full activation."""
    _, K, N = C5
    rng = np.random.default_rng(seed)
    w = normal(rng, (N, K), 0.02)
    x = normal(rng, (M, K))          # a prefix of the stream: the first M rows of the full x
    return x, w
