"""jax.random's threefry key operations on the device (csrc/random.cu), so the learner consumes
raw PRNG keys the way boonta's PPO does (boonta/algorithms/ppo.py:200, 230;
boonta/networks/distributions.py:21-23).

A key is two uint32 words (what jax.random.key_data returns); `key(seed)` makes the key of
jax.random.PRNGKey(seed). `partitionable` selects JAX's counter layout (True: the
jax_threefry_partitionable layout, the default of current JAX).
"""
from __future__ import annotations

import ctypes as C

import numpy as np
import torch

from . import _lib

_KIND = {"bits": 0, "uniform": 1, "normal": 2}


def key(seed: int) -> np.ndarray:
    seed = int(seed)
    if seed < 0:
        raise ValueError("key: non-negative seeds only")
    return np.array([(seed >> 32) & 0xFFFFFFFF, seed & 0xFFFFFFFF], np.uint32)


def as_key(k) -> np.ndarray:
    """An int seed, or two uint32 words (numpy, torch, list), as a key."""
    if isinstance(k, (int, np.integer)):
        return key(int(k))
    if isinstance(k, torch.Tensor):
        k = k.detach().cpu().numpy()
    k = np.asarray(k).reshape(-1)
    if k.size == 1:
        return key(int(k[0]))
    if k.size != 2:
        raise ValueError(f"a threefry key has two uint32 words, got {k.size}")
    return k.astype(np.uint32)


def _ckey(k):
    k = as_key(k)
    return (C.c_uint32 * 2)(int(k[0]), int(k[1]))


def split(k, num: int = 2, partitionable: bool = True) -> np.ndarray:
    out = (C.c_uint32 * (2 * num))()
    _lib.check(_lib.lib().bt_random_split(_ckey(k), num, int(partitionable), out))
    return np.array(out[:], np.uint32).reshape(num, 2)


def _fill(k, shape, kind, minval, maxval, partitionable, device):
    shape = tuple(shape)
    n = int(np.prod(shape)) if shape else 1
    out = torch.empty(shape, dtype=torch.int32 if kind == "bits" else torch.float32, device=device)
    _lib.check(_lib.lib().bt_random_fill(
        _ckey(k), n, _KIND[kind], float(minval), float(maxval), int(partitionable),
        out.data_ptr() if n else None, torch.cuda.current_stream(device).cuda_stream))
    return out


def bits(k, shape, device="cuda", partitionable: bool = True) -> torch.Tensor:
    """jax.random.bits(key, shape, uint32), as int32 storage of the same words."""
    return _fill(k, shape, "bits", 0.0, 0.0, partitionable, device)


def uniform(k, shape, minval=0.0, maxval=1.0, device="cuda", partitionable: bool = True):
    return _fill(k, shape, "uniform", minval, maxval, partitionable, device)


def normal(k, shape, device="cuda", partitionable: bool = True) -> torch.Tensor:
    return _fill(k, shape, "normal", 0.0, 0.0, partitionable, device)


def permutation(k, n: int, device="cuda", partitionable: bool = True) -> torch.Tensor:
    """jax.random.permutation(key, n) as int32 on the device."""
    lib = _lib.lib()
    out = torch.empty(n, dtype=torch.int32, device=device)
    need = int(lib.bt_random_permutation_workspace(n))
    if need < 0:
        raise ValueError(f"permutation: n = {n} unsupported")
    ws = torch.empty(max(need, 1), dtype=torch.uint8, device=device)
    _lib.check(lib.bt_random_permutation(
        _ckey(k), n, int(partitionable), out.data_ptr() if n else None, ws.data_ptr(), need,
        torch.cuda.current_stream(device).cuda_stream))
    return out
