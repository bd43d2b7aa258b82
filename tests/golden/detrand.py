"""Deterministic, numpy-version-independent normal samples for fixtures and parity inputs.

splitmix64 (S. Vigna, public-domain reference algorithm) drives a Box–Muller transform in float64; the result is
rounded to bf16-representable fp32 values so the same tensor feeds both the fp32 and the bf16 paths exactly.
"""
from __future__ import annotations

import numpy as np

_M1 = np.uint64(0xBF58476D1CE4E5B9)
_M2 = np.uint64(0x94D049BB133111EB)
_GOLD = np.uint64(0x9E3779B97F4A7C15)


def _splitmix64(seed: int, n: int) -> np.ndarray:
    with np.errstate(over="ignore"):
        z = (np.uint64(seed) + _GOLD * np.arange(1, n + 1, dtype=np.uint64)).astype(np.uint64)
        z = (z ^ (z >> np.uint64(30))) * _M1
        z = (z ^ (z >> np.uint64(27))) * _M2
        z = z ^ (z >> np.uint64(31))
    return z


def normal(seed: int, shape, std: float = 1.0, bf16_exact: bool = True) -> np.ndarray:
    n = int(np.prod(shape))
    m = (n + 1) // 2
    bits = _splitmix64(seed, 2 * m)
    u1 = ((bits[0::2] >> np.uint64(11)).astype(np.float64) + 1.0) / 9007199254740993.0   # (0, 1]
    u2 = (bits[1::2] >> np.uint64(11)).astype(np.float64) / 9007199254740992.0           # [0, 1)
    r = np.sqrt(-2.0 * np.log(u1))
    z = np.concatenate([r * np.cos(2 * np.pi * u2), r * np.sin(2 * np.pi * u2)])[:n]
    x = (z * std).astype(np.float32).reshape(shape)
    if bf16_exact:
        u = x.view(np.uint32).astype(np.uint64)
        u = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16) << 16
        x = u.astype(np.uint32).view(np.float32).reshape(shape)
    return x


def uniform(seed: int, shape) -> np.ndarray:
    n = int(np.prod(shape))
    bits = _splitmix64(seed, n)
    return ((bits >> np.uint64(11)).astype(np.float64) / 9007199254740992.0).reshape(shape)
