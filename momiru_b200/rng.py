"""Seeded synthetic inputs: SplitMix64 uniform and Box-Muller normal, vectorised.

Same generator and draw order as the reference's host initialisers
(src/momiru/tensor_light/tensor.rs:1467-1500 randu/randn, 1809-1840
SplitMix64): uniform values are the high 24 bits of each word times 2^-24,
mapped affinely to [lo, hi); normals take (u1, u2) pairs, emit the cos value
then the sin value, and are scaled by sigma.
"""
from __future__ import annotations

import numpy as np

_GAMMA = np.uint64(0x9E3779B97F4A7C15)
_M1 = np.uint64(0xBF58476D1CE4E5B9)
_M2 = np.uint64(0x94D049BB133111EB)


def splitmix64(seed: int, n: int) -> np.ndarray:
    """The first n outputs of SplitMix64 started at `seed`."""
    with np.errstate(over="ignore"):
        state = np.uint64(seed) + _GAMMA * np.arange(1, n + 1, dtype=np.uint64)
        v = state
        v = (v ^ (v >> np.uint64(30))) * _M1
        v = (v ^ (v >> np.uint64(27))) * _M2
        return v ^ (v >> np.uint64(31))


_CHUNK = 1 << 20


def _units(seed: int, n: int) -> np.ndarray:
    """n unit floats; generated in chunks to keep temporaries cache-sized."""
    out = np.empty(n, dtype=np.float32)
    idx = np.arange(1, _CHUNK + 1, dtype=np.uint64)
    scale = np.float32(1.0 / 16777216.0)
    with np.errstate(over="ignore"):
        for start in range(0, n, _CHUNK):
            cnt = min(_CHUNK, n - start)
            v = np.uint64(seed) + _GAMMA * (idx[:cnt] + np.uint64(start))
            v ^= v >> np.uint64(30)
            v *= _M1
            v ^= v >> np.uint64(27)
            v *= _M2
            v ^= v >> np.uint64(31)
            v >>= np.uint64(40)
            np.multiply(v.astype(np.float32), scale, out=out[start:start + cnt])
    return out


def randu(shape, seed: int, lo: float = -1.0, hi: float = 1.0) -> np.ndarray:
    n = int(np.prod(shape))
    u = _units(seed, n)
    u *= np.float32(hi - lo)
    u += np.float32(lo)
    return u.reshape(shape)


def randn(shape, seed: int, sigma: float = 1.0) -> np.ndarray:
    n = int(np.prod(shape))
    pairs = (n + 1) // 2
    u = _units(seed, 2 * pairs).reshape(pairs, 2)
    u1 = np.float32(1.0) - u[:, 0]
    u2 = u[:, 1]
    radius = np.sqrt(np.float32(-2.0) * np.log(u1)).astype(np.float32)
    angle = (np.float32(6.2831855) * u2).astype(np.float32)
    out = np.empty((pairs, 2), dtype=np.float32)
    out[:, 0] = radius * np.cos(angle)
    out[:, 1] = radius * np.sin(angle)
    out = out.reshape(-1)[:n] * np.float32(sigma)
    return out.astype(np.float32).reshape(shape)
