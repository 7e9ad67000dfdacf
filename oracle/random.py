"""JAX's threefry-based random numbers, restated in numpy (test infrastructure only).

The block cipher is threefry2x32 with 20 rounds (Salmon et al., SC 2011; Random123): key schedule
(k0, k1, k0 ^ k1 ^ 0x1BD11BDA), five groups of four rounds (x0 += x1; x1 = rotl(x1, r);
x1 ^= x0) with rotations (13, 15, 26, 6) and (17, 29, 16, 24) alternating, key injection after
group i: x0 += ks[i % 3], x1 += ks[(i + 1) % 3] + i. The key-level operations follow jax.random
for threefry keys (used by boonta/algorithms/ppo.py:200, 230 and
boonta/networks/distributions.py:21-23): split, bits, uniform, normal and permutation, in the
partitionable counter layout (the default of current JAX) or the original one. jax is not
installed here; the block is pinned by the Random123 known-answer vectors and the original
layout by JAX's documented split of PRNGKey(0) (tests/test_random.py).
"""
from __future__ import annotations

import math

import numpy as np

_ROT = (13, 15, 26, 6, 17, 29, 16, 24)


def _rotl(v, r):
    return ((v << np.uint32(r)) | (v >> np.uint32(32 - r))).astype(np.uint32)


def threefry2x32(k0, k1, c0, c1):
    """(y0, y1) for uint32 arrays of counters c0, c1 under the key (k0, k1)."""
    with np.errstate(over="ignore"):
        ks = (np.uint32(k0), np.uint32(k1), np.uint32(k0) ^ np.uint32(k1) ^ np.uint32(0x1BD11BDA))
        x0 = (np.asarray(c0, np.uint32) + ks[0]).astype(np.uint32)
        x1 = (np.asarray(c1, np.uint32) + ks[1]).astype(np.uint32)
        for g in range(5):
            for r in range(4):
                x0 = (x0 + x1).astype(np.uint32)
                x1 = _rotl(x1, _ROT[(g & 1) * 4 + r])
                x1 = x1 ^ x0
            i = g + 1
            x0 = (x0 + ks[i % 3]).astype(np.uint32)
            x1 = (x1 + ks[(i + 1) % 3] + np.uint32(i)).astype(np.uint32)
    return x0, x1


def key(seed: int) -> np.ndarray:
    """jax.random.PRNGKey(seed) / key_data(jax.random.key(seed)) for a non-negative seed."""
    seed = int(seed)
    return np.array([(seed >> 32) & 0xFFFFFFFF, seed & 0xFFFFFFFF], np.uint32)


def bits(k, n: int, partitionable: bool = True) -> np.ndarray:
    i = np.arange(n, dtype=np.uint64)
    if partitionable:
        y0, y1 = threefry2x32(k[0], k[1], (i >> np.uint64(32)).astype(np.uint32),
                              i.astype(np.uint32))
        return y0 ^ y1
    m = (n + 1) // 2
    c = np.zeros(2 * m, np.uint32)
    c[:n] = np.arange(n, dtype=np.uint32)
    y0, y1 = threefry2x32(k[0], k[1], c[:m], c[m:])
    return np.concatenate([y0, y1])[:n]


def split(k, num: int = 2, partitionable: bool = True) -> np.ndarray:
    if partitionable:
        y0, y1 = threefry2x32(k[0], k[1], np.zeros(num, np.uint32), np.arange(num, dtype=np.uint32))
        return np.stack([y0, y1], axis=1)
    return bits(k, 2 * num, partitionable=False).reshape(num, 2)


def uniform(k, n: int, minval=0.0, maxval=1.0, partitionable: bool = True) -> np.ndarray:
    b = bits(k, n, partitionable)
    f = ((b >> np.uint32(9)) | np.uint32(0x3F800000)).view(np.float32) - np.float32(1.0)
    lo, hi = np.float32(minval), np.float32(maxval)
    return np.maximum(lo, (f * (hi - lo) + lo).astype(np.float32))


def normal(k, n: int, partitionable: bool = True) -> np.ndarray:
    from scipy.special import erfinv

    lo = np.nextafter(np.float32(-1.0), np.float32(0.0))
    u = uniform(k, n, lo, 1.0, partitionable)
    return (np.float32(np.sqrt(2.0)) * erfinv(u.astype(np.float64)).astype(np.float32)).astype(np.float32)


def permutation_rounds(n: int) -> int:
    return 0 if n <= 1 else int(math.ceil(3 * math.log(n) / math.log(2 ** 32 - 1)))


def permutation(k, n: int, partitionable: bool = True) -> np.ndarray:
    """jax.random.permutation(key, n): rounds of (key, sub) = split(key); stable sort of the
    values by bits(sub, n)."""
    x = np.arange(n, dtype=np.int32)
    k = np.asarray(k, np.uint32)
    for _ in range(permutation_rounds(n)):
        k, sub = split(k, 2, partitionable)
        order = np.argsort(bits(sub, n, partitionable), kind="stable")
        x = x[order]
    return x
