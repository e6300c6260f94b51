"""Deterministic synthetic inputs shared by the golden-fixture generator and the tests.

``normal(seed, shape)`` draws standard-normal values from a counter-based
generator (splitmix64 -> two uniforms -> Box-Muller), then rounds them to
float32, so the same seed gives the same values on any machine and any numpy
version without storing the inputs themselves. Queries follow the reference
benchmark's scaling: ``w ~ N(0, 1/D)`` (``bench/bench_operator.py:336-337``
normalises to unit norm; N(0, 1/D) has expected norm 1).
"""

from __future__ import annotations

import numpy as np

_GOLDEN = np.uint64(0x9E3779B97F4A7C15)
_M1 = np.uint64(0xBF58476D1CE4E5B9)
_M2 = np.uint64(0x94D049BB133111EB)


def _splitmix64(x: np.ndarray) -> np.ndarray:
    with np.errstate(over="ignore"):
        z = x + _GOLDEN
        z = (z ^ (z >> np.uint64(30))) * _M1
        z = (z ^ (z >> np.uint64(27))) * _M2
        return z ^ (z >> np.uint64(31))


def _uniform(seed: int, stream: int, n: int) -> np.ndarray:
    base = (np.uint64(seed) << np.uint64(40)) ^ (np.uint64(stream) << np.uint64(36))
    with np.errstate(over="ignore"):
        ctr = np.arange(n, dtype=np.uint64) + base
    bits = _splitmix64(ctr) >> np.uint64(11)
    return (bits.astype(np.float64) + 0.5) * (1.0 / 9007199254740992.0)  # (0, 1)


def normal(seed: int, shape, scale: float = 1.0) -> np.ndarray:
    """float32-exact standard normal values (returned as float64) times ``scale``."""
    n = int(np.prod(shape))
    u1 = _uniform(seed, 1, n)
    u2 = _uniform(seed, 2, n)
    z = np.sqrt(-2.0 * np.log(u1)) * np.cos(2.0 * np.pi * u2)
    return (z * scale).astype(np.float32).astype(np.float64).reshape(shape)


def case_inputs(n: int, b: int, t: int, d: int, seed: int, n_queries: int = 0):
    """``(v, w, g, queries)`` for one case: v ~ N(0,1), w ~ N(0,1/D),
    g ~ N(0,1), queries ~ N(0,1/D) (``[n_queries, D]``)."""
    v = normal(seed, (n, b, t, d))
    w = normal(seed + 1, (d,), scale=1.0 / np.sqrt(d))
    g = normal(seed + 2, (b, t, d))
    q = normal(seed + 3, (max(n_queries, 0), d), scale=1.0 / np.sqrt(d))
    return v, w, g, q
