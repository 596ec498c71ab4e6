"""Platform-independent seeded inputs for the golden fixtures and parity tests.

numpy's Generator streams and SIMD transcendental functions are not promised to be
bit-identical across versions and CPUs, so fixtures whose inputs are regenerated
rather than stored use this generator: splitmix64 counters -> uniform doubles ->
an Irwin-Hall (sum of 12 uniforms - 6) approximate normal.  Only integer ops and
float64 additions are involved, so every machine produces the same bits.
"""
from __future__ import annotations

import numpy as np

_M64 = np.uint64(0xFFFFFFFFFFFFFFFF)


def _splitmix64(x: np.ndarray) -> np.ndarray:
    with np.errstate(over="ignore"):
        z = x + np.uint64(0x9E3779B97F4A7C15)
        z = (z ^ (z >> np.uint64(30))) * np.uint64(0xBF58476D1CE4E5B9)
        z = (z ^ (z >> np.uint64(27))) * np.uint64(0x94D049BB133111EB)
        return z ^ (z >> np.uint64(31))


def uniform(shape, seed: int) -> np.ndarray:
    """Uniform [0, 1) doubles, deterministic in (shape, seed)."""
    n = int(np.prod(shape))
    ctr = np.arange(n, dtype=np.uint64) + np.uint64(seed) * np.uint64(0x100000001B3)
    bits = _splitmix64(ctr) >> np.uint64(11)
    return (bits.astype(np.float64) * (1.0 / 9007199254740992.0)).reshape(shape)


def normal(shape, seed: int) -> np.ndarray:
    """Approximately standard-normal doubles (Irwin-Hall of 12 uniforms)."""
    n = int(np.prod(shape))
    u = uniform((12, n), seed)
    return (u.sum(axis=0) - 6.0).reshape(shape)


def integers(shape, seed: int, high: int) -> np.ndarray:
    n = int(np.prod(shape))
    ctr = np.arange(n, dtype=np.uint64) + np.uint64(seed) * np.uint64(0x100000001B3)
    return (_splitmix64(ctr) % np.uint64(high)).astype(np.int64).reshape(shape)
