"""Deterministic, platform-independent inputs for the golden fixtures.

Values come from splitmix64 of (seed, index) turned into an approximately normal variate with exact
integer/float64 arithmetic (Irwin-Hall sum of four 24-bit uniforms, centred and scaled), so regenerating
an input anywhere gives the same bits without storing it.
"""

from __future__ import annotations

import numpy as np
import torch

_M64 = np.uint64(0xFFFFFFFFFFFFFFFF)


def _splitmix(x: np.ndarray) -> np.ndarray:
    with np.errstate(over="ignore"):
        x = x + np.uint64(0x9E3779B97F4A7C15)
        x = (x ^ (x >> np.uint64(30))) * np.uint64(0xBF58476D1CE4E5B9)
        x = (x ^ (x >> np.uint64(27))) * np.uint64(0x94D049BB133111EB)
        return x ^ (x >> np.uint64(31))


def uniforms(seed: int, n: int, lane: int = 0) -> np.ndarray:
    """n float64 values in [0, 1) with 24-bit resolution."""
    idx = np.arange(n, dtype=np.uint64) * np.uint64(4) + np.uint64(lane)
    with np.errstate(over="ignore"):
        h = _splitmix(idx ^ (np.uint64(seed) * np.uint64(0xD1B54A32D192ED03)))
    return (h >> np.uint64(40)).astype(np.float64) / float(1 << 24)


def normal(seed: int, shape, scale: float = 1.0, shift: float = 0.0) -> np.ndarray:
    """float64 approx N(shift, scale^2): (u1+u2+u3+u4 - 2) * sqrt(3)."""
    n = int(np.prod(shape))
    s = sum(uniforms(seed, n, lane) for lane in range(4))
    return ((s - 2.0) * 1.7320508075688772 * scale + shift).reshape(shape)


def bf16(seed: int, shape, scale: float = 1.0, shift: float = 0.0) -> torch.Tensor:
    """bf16 CPU tensor (round-to-nearest-even of the float64 value via float32)."""
    return torch.from_numpy(normal(seed, shape, scale, shift).astype(np.float32)).bfloat16()


def f32(seed: int, shape, scale: float = 1.0) -> torch.Tensor:
    return torch.from_numpy(normal(seed, shape, scale).astype(np.float32))


def permutation(seed: int, n: int) -> np.ndarray:
    """A deterministic permutation of range(n) (argsort of hashed keys)."""
    keys = _splitmix(np.arange(n, dtype=np.uint64) ^ (np.uint64(seed) << np.uint64(32)))
    return np.argsort(keys, kind="stable").astype(np.int64)
