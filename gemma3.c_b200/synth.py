"""Seeded synthetic inputs for the attention hot path.

Counter-based generator: element i of stream `seed` is derived from
splitmix64(seed, i), and normals come from the Box-Muller transform of two
24-bit uniforms, so any slice of any stream is reproducible without
generating its prefix.  BF16 weights are made by truncating fp32 draws, the
way the reference converts fp32 to BF16 (gemma3_kernels.h:279-283).
"""
from __future__ import annotations

import numpy as np

_M64 = np.uint64(0xFFFFFFFFFFFFFFFF)


def _splitmix64(x: np.ndarray) -> np.ndarray:
    with np.errstate(over="ignore"):
        x = x + np.uint64(0x9E3779B97F4A7C15)
        x = (x ^ (x >> np.uint64(30))) * np.uint64(0xBF58476D1CE4E5B9)
        x = (x ^ (x >> np.uint64(27))) * np.uint64(0x94D049BB133111EB)
        return x ^ (x >> np.uint64(31))


def normal(seed: int, shape, std: float = 1.0, mean: float = 0.0) -> np.ndarray:
    """fp32 N(mean, std^2) array of the given shape from stream `seed`."""
    n = int(np.prod(shape))
    half = (n + 1) // 2
    with np.errstate(over="ignore"):
        base = np.uint64(seed) * np.uint64(0xD1B54A32D192ED03)
        r = _splitmix64(base + np.arange(half, dtype=np.uint64))
    u1 = ((r >> np.uint64(40)).astype(np.float64) + 0.5) / 16777216.0
    u2 = (r & np.uint64(0xFFFFFF)).astype(np.float64) / 16777216.0
    rad = np.sqrt(-2.0 * np.log(u1))
    z = np.empty(2 * half, dtype=np.float64)
    z[0::2] = rad * np.cos(2 * np.pi * u2)
    z[1::2] = rad * np.sin(2 * np.pi * u2)
    return (z[:n] * std + mean).astype(np.float32).reshape(shape)


def uniform_int(seed: int, n: int, hi: int) -> np.ndarray:
    """n integers uniform in [0, hi)."""
    with np.errstate(over="ignore"):
        r = _splitmix64(np.uint64(seed) * np.uint64(0xA24BAED4963EE407) + np.arange(n, dtype=np.uint64))
    return (r % np.uint64(hi)).astype(np.int64)


def bf16_trunc(x: np.ndarray) -> np.ndarray:
    """fp32 -> BF16 bit pattern (uint16) by truncation, as the reference does."""
    return (np.ascontiguousarray(x, dtype=np.float32).view(np.uint32) >> 16).astype(np.uint16)


def bf16_to_f32(h: np.ndarray) -> np.ndarray:
    return (h.astype(np.uint32) << 16).view(np.float32)


def qk_norm_gains(seed: int) -> tuple[np.ndarray, np.ndarray]:
    """Stored q/k-norm weights w ~ N(0, 0.1) as BF16; the kernels apply 1+w
    (gemma3_kernels.c:301), giving effective gains ~ 1 + N(0, 0.1)."""
    return bf16_trunc(normal(seed, (256,), 0.1)), bf16_trunc(normal(seed + 1, (256,), 0.1))
