"""CUDA GAE (bt_gae) parity: the reference's known-answer vectors, bit-exact agreement with the
oracle's restatement of the kernel's chunked order, and the reference's sequential order within
1e-5 relative (plus 1e-6 of the advantages' scale: the chunks compose partial sums, so an
advantage near zero carries the rounding of its larger neighbours), edge shapes."""
from pathlib import Path

import numpy as np
import pytest

GOLDEN = Path(__file__).parent / "golden" / "gae_kat.npz"
pytestmark = pytest.mark.gpu


def _run(reward, term, trunc, values, boot, gamma, lam, rho=None, c=None):
    import torch

    from boonta_b200.learner import gae

    t = lambda x, dt: torch.as_tensor(np.ascontiguousarray(x), dtype=dt, device="cuda")
    adv, ret = gae(t(reward, torch.float32), t(term, torch.uint8), t(trunc, torch.uint8),
                   t(values, torch.float32), t(boot, torch.float32), gamma, lam,
                   rho=None if rho is None else t(rho, torch.float32),
                   c=None if c is None else t(c, torch.float32))
    torch.cuda.synchronize()
    return adv.cpu().numpy(), ret.cpu().numpy()


@pytest.mark.parametrize("case", ["gae", "vtrace"])
def test_cuda_gae_matches_the_reference_known_answers(case):
    d = np.load(GOLDEN)
    g = lambda k: d[f"{case}/{k}"]
    args = (g("reward"), g("terminated"), g("truncated"), g("values"), g("bootstrap"),
            float(d["gamma"]), float(d["gae_lambda"]))
    adv, ret = _run(*args, rho=g("rho"), c=g("c"))
    scale = max(1.0, float(np.abs(g("advantages")).max()))
    np.testing.assert_allclose(adv, g("advantages"), rtol=1e-5, atol=1e-6 * scale)
    np.testing.assert_allclose(ret, g("returns"), rtol=1e-5, atol=1e-6 * scale)
    if case == "gae":  # rho = c = 1 also through the default (NULL weights) path
        adv2, _ = _run(*args)
        np.testing.assert_array_equal(adv2, adv)


# chunks of 1 to 188 steps (kept in registers up to 16), ragged column blocks, the five configs'
# shapes
SHAPES = [(1, 1), (7, 5), (3, 33), (128, 16), (64, 8192), (128, 4096), (64, 4096), (33, 96),
          (500, 64), (512, 48), (513, 32), (16, 9728), (1500, 16), (2, 48)]


@pytest.mark.parametrize("shape", SHAPES, ids=[f"{t}x{n}" for t, n in SHAPES])
@pytest.mark.parametrize("weighted", [False, True], ids=["gae", "vtrace"])
def test_cuda_gae_is_bit_exact_with_the_oracle_order(shape, weighted):
    from oracle.gae import gae, gae_chunked

    rng = np.random.default_rng(hash(shape) % 2**32)
    t, n = shape
    reward = rng.standard_normal(shape).astype(np.float32)
    values = rng.standard_normal(shape).astype(np.float32)
    boot = rng.standard_normal(n).astype(np.float32)
    term = (rng.random(shape) < 0.05).astype(np.uint8)
    trunc = ((rng.random(shape) < 0.05) & (term == 0)).astype(np.uint8)
    rho = rng.uniform(0.5, 1.5, shape).astype(np.float32) if weighted else None
    c = rng.uniform(0.5, 1.5, shape).astype(np.float32) if weighted else None
    gamma, lam = 0.97, 0.95
    adv, ret = _run(reward, term, trunc, values, boot, gamma, lam, rho, c)
    ea, er = gae_chunked(reward, term, trunc, values, boot, gamma, lam, rho=rho, c=c)
    np.testing.assert_array_equal(adv, ea)
    np.testing.assert_array_equal(ret, er)
    sa, sr = gae(reward, term, trunc, values, boot, gamma, lam, rho=rho, c=c)
    scale = max(1.0, float(np.abs(sa).max()))
    np.testing.assert_allclose(adv, sa, rtol=1e-5, atol=1e-6 * scale)
    np.testing.assert_allclose(ret, sr, rtol=1e-5, atol=1e-6 * scale)


def test_cuda_gae_empty_inputs():
    import torch

    from boonta_b200.learner import gae

    z = torch.zeros((0, 4), device="cuda")
    adv, ret = gae(z, z.to(torch.uint8), z.to(torch.uint8), z, torch.zeros(4, device="cuda"), 0.9, 0.9)
    assert adv.shape == (0, 4)
