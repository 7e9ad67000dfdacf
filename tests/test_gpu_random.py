"""Device random numbers (csrc/random.cu, boonta_b200.random) against the numpy restatement of
jax.random's threefry operations (oracle/random.py): raw blocks, bits, uniform and permutations
bit for bit in both counter layouts, normals within float32 rounding (CUDA's erfinvf against
scipy's double erfinv), edge sizes, and the PPO API drawing from them."""
import numpy as np
import pytest

from oracle import random as orand

pytestmark = pytest.mark.gpu

SIZES = [0, 1, 2, 3, 1000, 4097, 262_144]


def test_device_blocks_match_the_known_answers_and_the_oracle():
    import ctypes as C

    import torch

    from boonta_b200 import _lib

    rng = np.random.default_rng(0)
    c0 = rng.integers(0, 2 ** 32, 5000, dtype=np.uint64).astype(np.uint32)
    c1 = rng.integers(0, 2 ** 32, 5000, dtype=np.uint64).astype(np.uint32)
    c0[:3] = [0, 0xFFFFFFFF, 0x243F6A88]
    c1[:3] = [0, 0xFFFFFFFF, 0x85A308D3]
    t = lambda x: torch.tensor(x.astype(np.int64), device="cuda").to(torch.int32)
    y0, y1 = torch.empty(5000, dtype=torch.int32, device="cuda"), torch.empty(5000, dtype=torch.int32, device="cuda")
    d0, d1 = t(c0), t(c1)
    for key in ((0, 0), (0x13198A2E, 0x03707344)):
        _lib.check(_lib.lib().bt_threefry2x32(key[0], key[1], d0.data_ptr(), d1.data_ptr(),
                                              y0.data_ptr(), y1.data_ptr(), 5000, None))
        torch.cuda.synchronize()
        e0, e1 = orand.threefry2x32(key[0], key[1], c0, c1)
        np.testing.assert_array_equal(y0.cpu().numpy().view(np.uint32), e0)
        np.testing.assert_array_equal(y1.cpu().numpy().view(np.uint32), e1)
    assert int(y0[2].item()) & 0xFFFFFFFF == 0xC4923A9C  # Random123 known answer


@pytest.mark.parametrize("n", SIZES)
@pytest.mark.parametrize("partitionable", [True, False])
def test_bits_uniform_normal_permutation(n, partitionable):
    import torch

    from boonta_b200 import random as trandom

    k = orand.key(42 + n)
    b = trandom.bits(k, (n,), partitionable=partitionable)
    u = trandom.uniform(k, (n,), np.finfo(np.float32).tiny, 1.0, partitionable=partitionable)
    z = trandom.normal(k, (n,), partitionable=partitionable)
    p = trandom.permutation(k, n, partitionable=partitionable)
    torch.cuda.synchronize()
    np.testing.assert_array_equal(b.cpu().numpy().view(np.uint32), orand.bits(k, n, partitionable))
    np.testing.assert_array_equal(u.cpu().numpy(), orand.uniform(k, n, np.finfo(np.float32).tiny,
                                                                 1.0, partitionable))
    np.testing.assert_allclose(z.cpu().numpy(), orand.normal(k, n, partitionable), rtol=2e-6,
                               atol=2e-6)
    np.testing.assert_array_equal(p.cpu().numpy(), orand.permutation(k, n, partitionable))


def test_permutation_rejects_a_short_workspace():
    import ctypes as C

    import torch

    from boonta_b200 import _lib

    out = torch.empty(1000, dtype=torch.int32, device="cuda")
    key = (C.c_uint32 * 2)(0, 1)
    with pytest.raises(RuntimeError, match="workspace"):
        _lib.check(_lib.lib().bt_random_permutation(key, 1000, 1, out.data_ptr(), None, 0, None))


def test_ppo_update_draws_the_reference_permutations():
    from boonta_b200 import configs
    from boonta_b200.ppo import PPO

    w = configs.make("c1").scaled(num_steps=8, num_envs=16, num_minibatches=2, update_epochs=3)
    ppo = PPO(w.ppo, w.network, w.optimizer)
    perms = ppo._permutations(11, 128, "cuda").cpu().numpy()
    keys = orand.split(orand.key(11), 3)
    for e in range(3):
        np.testing.assert_array_equal(perms[e], orand.permutation(keys[e], 128))
