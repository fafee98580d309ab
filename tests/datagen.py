"""Seeded synthetic inputs shaped like the benchmark configurations.

numpy's PCG64 generator stands in for the PCG32 streams named in the
benchmark plan; every generator takes an explicit seed.
"""
from __future__ import annotations

import numpy as np

from oracle.oracle import NP_DTYPE, NP_UINT

KEY_TYPES = ["u8", "i8", "u16", "i16", "u32", "i32", "u64", "i64", "f32", "f64"]


def uniform_bits(kt: str, n: int, seed: int) -> np.ndarray:
    """Keys uniform over every bit pattern of the type (floats include NaNs/infs)."""
    dt = np.dtype(NP_DTYPE[kt])
    rng = np.random.default_rng(seed)
    raw = rng.integers(0, 256, size=n * dt.itemsize, dtype=np.uint8)
    return raw.view(dt).copy()


def low_entropy(kt: str, n: int, seed: int) -> np.ndarray:
    """Bitwise AND of three uniform words: P(bit = 1) = 1/8."""
    dt = np.dtype(NP_DTYPE[kt])
    u = NP_UINT[dt.itemsize]
    a, b, c = (uniform_bits(kt, n, seed + i).view(u) for i in range(3))
    return (a & b & c).view(dt).copy()


def special_floats(kt: str, n: int, seed: int, scale: float = 1e3, frac: float = 0.001) -> np.ndarray:
    """N(0, scale) with frac each of -0.0, +0.0, +inf, -inf and quiet NaN at random positions."""
    dt = np.dtype(NP_DTYPE[kt])
    rng = np.random.default_rng(seed)
    x = (rng.standard_normal(n) * scale).astype(dt)
    specials = [-0.0, 0.0, np.inf, -np.inf, np.nan]
    m = max(1, int(n * frac)) if n >= 10 else 0
    for s in specials:
        if m:
            idx = rng.integers(0, n, size=m)
            x[idx] = dt.type(s)
    return x


def zipf_table(kt: str, n: int, seed: int, distinct: int = 65536, s: float = 1.1, below: int | None = None):
    """Zipf(s) draws over a seeded table of `distinct` values (optionally < 2**below)."""
    dt = np.dtype(NP_DTYPE[kt])
    rng = np.random.default_rng(seed)
    table = uniform_bits(kt, distinct, seed + 1000).view(NP_UINT[dt.itemsize]).copy()
    if below is not None:
        table = table % np.array(1 << below, dtype=table.dtype)
    ranks = np.arange(1, distinct + 1, dtype=np.float64)
    p = ranks ** (-s)
    p /= p.sum()
    draws = rng.choice(distinct, size=n, p=p)
    return table[draws].view(dt).copy()


def values_for(n: int, value_bytes: int, seed: int = 0) -> np.ndarray:
    """Payloads carrying the original index, so stability is visible."""
    idx = np.arange(n, dtype=np.uint64)
    if value_bytes == 16:
        v = np.empty((n, 2), dtype=np.uint64)
        v[:, 0] = idx
        v[:, 1] = ~idx
        return v
    return idx.astype(NP_UINT[value_bytes])
