"""Philox4x32-10 Gumbel noise, restated in numpy — TEST INFRASTRUCTURE ONLY.

The reference draws its sampling noise per slot with ``torch.rand`` and maps it
to Gumbel noise as ``-log(-log(clamp(u, 1e-8, 1)))``
(engine/backend/executor.py:1229-1253, ``_build_sampling_noise``).  The B200
backend draws the uniform variate in-kernel from the counter-based generator
Philox4x32-10 (Salmon, Moraes, Dror, Shaw: "Parallel random numbers: as easy as
1, 2, 3", SC'11), keyed by the engine seed, with the counter
``(rank j, 16 * frame + stage, key lo, key hi)``.  This module restates that
generator from the paper and the reference's transform so tests can check the
device's noise value by value and its distribution.
"""

from __future__ import annotations

import numpy as np

_M0, _M1 = np.uint64(0xD2511F53), np.uint64(0xCD9E8D57)
_W0, _W1 = np.uint32(0x9E3779B9), np.uint32(0xBB67AE85)
_MASK = np.uint64(0xFFFFFFFF)


def philox4x32_10(c0, c1, c2, c3, k0, k1):
    """Ten Philox rounds on uint32 arrays; returns the four output words."""
    c0, c1, c2, c3 = (np.asarray(v, dtype=np.uint32) for v in (c0, c1, c2, c3))
    k0 = np.asarray(k0, dtype=np.uint32).copy()
    k1 = np.asarray(k1, dtype=np.uint32).copy()
    with np.errstate(over="ignore"):
        for _ in range(10):
            p0 = _M0 * c0.astype(np.uint64)
            p1 = _M1 * c2.astype(np.uint64)
            hi0, lo0 = (p0 >> np.uint64(32)).astype(np.uint32), (p0 & _MASK).astype(np.uint32)
            hi1, lo1 = (p1 >> np.uint64(32)).astype(np.uint32), (p1 & _MASK).astype(np.uint32)
            c0, c1, c2, c3 = hi1 ^ c1 ^ k0, lo1, hi0 ^ c3 ^ k1, lo0
            k0 = k0 + _W0
            k1 = k1 + _W1
    return c0, c1, c2, c3


def uniform(seed: int, keys, frames, stage: int, cols: int) -> np.ndarray:
    """fp32 u in (0, 1) of shape [R, cols] for per-row keys (int64) and frame counters."""
    keys = np.asarray(keys, dtype=np.int64).astype(np.uint64)
    frames = np.asarray(frames, dtype=np.int64)
    R = keys.shape[0]
    j = np.broadcast_to(np.arange(cols, dtype=np.uint32)[None, :], (R, cols))
    step = np.broadcast_to(((frames * 16 + stage) & 0xFFFFFFFF).astype(np.uint32)[:, None], (R, cols))
    klo = np.broadcast_to((keys & _MASK).astype(np.uint32)[:, None], (R, cols))
    khi = np.broadcast_to((keys >> np.uint64(32)).astype(np.uint32)[:, None], (R, cols))
    seed = int(seed) & ((1 << 64) - 1)
    r0, _, _, _ = philox4x32_10(j, step, klo, khi, np.uint32(seed & 0xFFFFFFFF), np.uint32(seed >> 32))
    # ((float)r + 0.5f) * 2^-32 in fp32, each operation rounded to nearest
    u = (r0.astype(np.float32) + np.float32(0.5)) * np.float32(2.3283064365386963e-10)
    return u.astype(np.float32)


def gumbel(seed: int, keys, frames, stage: int, cols: int = 50) -> np.ndarray:
    """executor.py:1238-1251's transform of the Philox uniforms, in fp32."""
    u = np.clip(uniform(seed, keys, frames, stage, cols), np.float32(1e-8), np.float32(1.0))
    return (-np.log(-np.log(u))).astype(np.float32)
