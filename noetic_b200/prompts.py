"""Seeded synthetic prompts: stream s draws its ids from Rng::new(base + s)
with Rng::below(vocab) (rng.rs:25-38, 46-56, 75-90), vectorised over
streams with numpy (uint64 arithmetic wraps like Rust's wrapping ops)."""

from __future__ import annotations

import numpy as np

_M = np.uint64


def _splitmix(z):
    z = z + _M(0x9E3779B97F4A7C15)
    r = z
    r = (r ^ (r >> _M(30))) * _M(0xBF58476D1CE4E5B9)
    r = (r ^ (r >> _M(27))) * _M(0x94D049BB133111EB)
    return z, r ^ (r >> _M(31))


def rng_states(seeds: np.ndarray) -> np.ndarray:
    """Rng::new for every seed: [n, 4] uint64."""
    with np.errstate(over="ignore"):
        z = np.asarray(seeds, dtype=np.uint64) ^ _M(0xA0761D6478BD642F)
        out = np.empty((z.size, 4), dtype=np.uint64)
        for i in range(4):
            z, out[:, i] = _splitmix(z)
        zero = ~out.any(axis=1)
        out[zero, 0] = _M(0x9E3779B97F4A7C15)
    return out


def _rotl(x, k):
    return (x << _M(k)) | (x >> _M(64 - k))


def next_u64(s: np.ndarray) -> np.ndarray:
    """xoshiro256++ step on every row of s [n, 4] (in place); returns outputs."""
    with np.errstate(over="ignore"):
        s0, s1, s2, s3 = s[:, 0].copy(), s[:, 1].copy(), s[:, 2].copy(), s[:, 3].copy()
        result = _rotl(s0 + s3, 23) + s0
        t = s1 << _M(17)
        s2 ^= s0
        s3 ^= s1
        s1 ^= s2
        s0 ^= s3
        s2 ^= t
        s3 = _rotl(s3, 45)
        s[:, 0], s[:, 1], s[:, 2], s[:, 3] = s0, s1, s2, s3
    return result


def below(s: np.ndarray, n: int) -> np.ndarray:
    """Rng::below(n) on every row (Lemire threshold rejection, then modulo)."""
    if n == 1:
        return np.zeros(s.shape[0], dtype=np.uint64)
    bound = _M(n)
    threshold = _M(((1 << 64) - n) % n)
    out = np.empty(s.shape[0], dtype=np.uint64)
    pending = np.arange(s.shape[0])
    while pending.size:
        sub = s[pending]
        r = next_u64(sub)
        s[pending] = sub
        ok = r >= threshold
        out[pending[ok]] = r[ok] % bound
        pending = pending[~ok]
    return out


def uniform_prompts(n_streams: int, length: int, vocab: int, base_seed: int, first: int = 0) -> np.ndarray:
    """[n_streams, length] uint32 ids; stream i uses Rng::new(base_seed + first + i)."""
    seeds = np.arange(first, first + n_streams, dtype=np.uint64) + _M(base_seed)
    s = rng_states(seeds)
    ids = np.empty((n_streams, length), dtype=np.uint32)
    for t in range(length):
        ids[:, t] = below(s, vocab).astype(np.uint32)
    return ids
