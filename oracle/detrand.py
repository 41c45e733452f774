"""Version-independent seeded random streams for test inputs (test infrastructure only).

Every value is a pure function of (seed, index): SplitMix64 (Steele, Lea & Flood,
"Fast splittable pseudorandom number generators", OOPSLA 2014) gives 64 random bits
per index, and the Box-Muller transform turns pairs of uniforms into normals.  Test
fixtures that store only a seed therefore regenerate the same inputs on any machine
and with any numpy version.
"""
from __future__ import annotations

import numpy as np

_GOLDEN = np.uint64(0x9E3779B97F4A7C15)
_M1 = np.uint64(0xBF58476D1CE4E5B9)
_M2 = np.uint64(0x94D049BB133111EB)


def splitmix64(seed: int, n: int, offset: int = 0) -> np.ndarray:
    with np.errstate(over="ignore"):
        i = np.arange(offset, offset + n, dtype=np.uint64) + np.uint64(1)
        z = np.uint64(seed & 0xFFFFFFFFFFFFFFFF) + i * _GOLDEN
        z = (z ^ (z >> np.uint64(30))) * _M1
        z = (z ^ (z >> np.uint64(27))) * _M2
        return z ^ (z >> np.uint64(31))


def uniform(seed: int, n: int, offset: int = 0) -> np.ndarray:
    """Uniform float64 in (0, 1]."""
    z = splitmix64(seed, n, offset)
    return ((z >> np.uint64(11)).astype(np.float64) + 1.0) * (1.0 / 9007199254740992.0)


def normal(seed: int, shape, std: float = 1.0, dtype=np.float32) -> np.ndarray:
    n = int(np.prod(shape))
    m = (n + 1) // 2
    u1 = uniform(seed, m, 0)
    u2 = uniform(seed ^ 0x5DEECE66D, m, 0)
    r = np.sqrt(-2.0 * np.log(u1))
    t = 2.0 * np.pi * u2
    z = np.empty(2 * m, dtype=np.float64)
    z[0::2] = r * np.cos(t)
    z[1::2] = r * np.sin(t)
    return (z[:n] * std).astype(dtype).reshape(shape)


def integers(seed: int, n: int, lo: int, hi: int) -> np.ndarray:
    """Integers uniform in [lo, hi] (inclusive)."""
    span = np.uint64(hi - lo + 1)
    return (splitmix64(seed, n) % span).astype(np.int64) + lo


def permutation(seed: int, n: int) -> np.ndarray:
    return np.argsort(splitmix64(seed, n), kind="stable")
