"""The threefry random numbers (bt_threefry2x32_host, bt_random_split; csrc/random.cu) and their
numpy restatement (oracle/random.py) against published known answers, on the CPU: the Random123
threefry2x32-20 vectors and JAX's documented split of PRNGKey(0) in its original counter layout."""
import ctypes as C

import numpy as np
import pytest

from oracle import random as orand

# Random123 kat_vectors, threefry2x32 with 20 rounds: (counter, key) -> output
KAT = [((0x00000000, 0x00000000), (0x00000000, 0x00000000), (0x6B200159, 0x99BA4EFE)),
       ((0xFFFFFFFF, 0xFFFFFFFF), (0xFFFFFFFF, 0xFFFFFFFF), (0x1CB996FC, 0xBB002BE7)),
       ((0x243F6A88, 0x85A308D3), (0x13198A2E, 0x03707344), (0xC4923A9C, 0x483DF7A0))]
# jax.random.split(jax.random.PRNGKey(0)) with the original counter layout
SPLIT0 = [[4146024105, 967050713], [2718843009, 1272950319]]


def _lib():
    from boonta_b200 import _lib

    return _lib.lib()


@pytest.mark.parametrize("ctr,key,out", KAT)
def test_threefry_known_answers(ctr, key, out):
    y = (C.c_uint32 * 2)()
    _lib().bt_threefry2x32_host(key[0], key[1], ctr[0], ctr[1], y)
    assert (y[0], y[1]) == out
    o0, o1 = orand.threefry2x32(key[0], key[1], np.array([ctr[0]]), np.array([ctr[1]]))
    assert (int(o0[0]), int(o1[0])) == out


def test_original_layout_split_matches_jax():
    k = orand.key(0)
    np.testing.assert_array_equal(orand.split(k, 2, partitionable=False), SPLIT0)
    out = (C.c_uint32 * 4)()
    kk = (C.c_uint32 * 2)(*k)
    _lib().bt_random_split(kk, 2, 0, out)
    assert [[out[0], out[1]], [out[2], out[3]]] == SPLIT0


@pytest.mark.parametrize("partitionable", [True, False])
def test_library_split_matches_the_oracle(partitionable):
    rng = np.random.default_rng(1)
    for _ in range(5):
        k = rng.integers(0, 2 ** 32, 2, dtype=np.uint64).astype(np.uint32)
        num = int(rng.integers(1, 9))
        out = (C.c_uint32 * (2 * num))()
        _lib().bt_random_split((C.c_uint32 * 2)(*k), num, int(partitionable), out)
        np.testing.assert_array_equal(np.array(out[:], np.uint32).reshape(num, 2),
                                      orand.split(k, num, partitionable))


def test_permutation_oracle_is_a_permutation_with_jaxs_round_count():
    assert orand.permutation_rounds(1) == 0
    assert orand.permutation_rounds(2 ** 16) == 2
    assert orand.permutation_rounds(262_144) == 2
    p = orand.permutation(orand.key(3), 1000)
    assert sorted(p.tolist()) == list(range(1000))
    assert not np.array_equal(p, np.arange(1000))
    np.testing.assert_array_equal(orand.permutation(orand.key(3), 1), [0])


def test_uniform_bit_trick_stays_in_range():
    u = orand.uniform(orand.key(7), 100_000, np.finfo(np.float32).tiny, 1.0)
    assert u.min() >= np.finfo(np.float32).tiny and u.max() < 1.0
    assert abs(float(u.mean()) - 0.5) < 0.01


def test_python_keys_and_host_split():
    import torch

    from boonta_b200 import random as trandom

    np.testing.assert_array_equal(trandom.key(0), [0, 0])
    np.testing.assert_array_equal(trandom.key(2 ** 32 + 5), [1, 5])
    np.testing.assert_array_equal(trandom.as_key(7), trandom.key(7))
    np.testing.assert_array_equal(trandom.as_key(torch.tensor([7])), trandom.key(7))
    np.testing.assert_array_equal(trandom.as_key([3, 4]), np.array([3, 4], np.uint32))
    with pytest.raises(ValueError):
        trandom.as_key([1, 2, 3])
    with pytest.raises(ValueError):
        trandom.key(-1)
    # split on the host through the library, both layouts, against the oracle
    for part in (True, False):
        np.testing.assert_array_equal(trandom.split(7, 5, part), orand.split(orand.key(7), 5, part))
