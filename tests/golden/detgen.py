"""Deterministic, platform-independent synthetic inputs for fixtures and tests.

Values come from a counter-based integer hash (splitmix64), so the same
(seed, shape) gives bit-identical arrays on any machine and any numpy version:
the golden fixtures store only outputs, and the tests regenerate the inputs.

det_normal: Irwin-Hall sum of four 16-bit uniforms, rescaled to unit variance
(support [-3.46, 3.46]); every step is exact or a single IEEE rounding.
"""
from __future__ import annotations

import numpy as np

_M1 = np.uint64(0xBF58476D1CE4E5B9)
_M2 = np.uint64(0x94D049BB133111EB)
_GOLD = np.uint64(0x9E3779B97F4A7C15)


def splitmix64(x: np.ndarray) -> np.ndarray:
    with np.errstate(over="ignore"):
        z = (np.asarray(x, dtype=np.uint64) + _GOLD).astype(np.uint64)
        z = (z ^ (z >> np.uint64(30))) * _M1
        z = (z ^ (z >> np.uint64(27))) * _M2
        return z ^ (z >> np.uint64(31))


def det_bits(seed: int, n: int) -> np.ndarray:
    key = splitmix64(np.array([seed], dtype=np.uint64))[0]
    return splitmix64(np.arange(n, dtype=np.uint64) ^ key)


def det_normal(seed: int, shape, scale: float = 1.0) -> np.ndarray:
    n = int(np.prod(shape))
    x = det_bits(seed, n)
    acc = np.zeros(n, dtype=np.float64)
    for k in range(4):
        acc += ((x >> np.uint64(16 * k)) & np.uint64(0xFFFF)).astype(np.float64) + 0.5
    z = (acc / 65536.0 - 2.0) * 1.7320508075688772
    return (z * scale).astype(np.float32).reshape(shape)


def det_ints(seed: int, n: int, lo: int, hi: int) -> np.ndarray:
    """n integers uniform in [lo, hi] (inclusive)."""
    x = det_bits(seed, n)
    return (lo + (x % np.uint64(hi - lo + 1)).astype(np.int64)).astype(np.int64)


def det_perm(seed: int, n: int) -> np.ndarray:
    return np.argsort(det_bits(seed, n), kind="stable").astype(np.int64)


def det_outlier_mask(seed: int, shape, frac: float) -> np.ndarray:
    x = det_bits(seed, int(np.prod(shape)))
    return ((x >> np.uint64(11)).astype(np.float64) / float(1 << 53) < frac).reshape(shape)
