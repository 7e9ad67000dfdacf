"""The linear-scan oracle (oracle/scan.py) against the float64 recurrence and its own
gradient, on the cases the reference's tests use (tests/test_networks.py:129-210)."""
import numpy as np

from oracle import scan as osc
from oracle.network import bf16_round


def problem(seed, shape=(4, 16, 128)):
    rng = np.random.default_rng(seed)
    a = (rng.uniform(size=shape) * 0.9 + 0.05).astype(np.float32)
    b = rng.uniform(size=shape).astype(np.float32)
    init = rng.standard_normal((shape[0], shape[2])).astype(np.float32)
    return a, b, init


def test_sequential_and_chunked_orders_match_the_exact_recurrence():
    # tests/test_networks.py:141-149: every scan within 1e-5 of the reference
    a, b, init = problem(3)
    exact = osc.exact(a, b, init)
    for out in (osc.sequential(a, b, init), osc.chunked(a, b, init)):
        np.testing.assert_allclose(out, exact, atol=1e-5)


def test_backward_matches_finite_differences_of_the_exact_recurrence():
    # the custom VJP (scan.py:81-87) against d/dx of sum(weight * scan(x)) in float64
    a, b, init = problem(4, (2, 9, 5))
    w = np.random.default_rng(5).standard_normal(a.shape)
    h = osc.sequential(a, b, init)
    x0 = [x.astype(np.float64) for x in (a, b, init)]

    def loss(args):
        return float((w * osc.exact(*args)).sum())

    eps = 1e-6
    numeric = []
    for k in range(3):
        num = np.zeros_like(x0[k])
        for idx in np.ndindex(num.shape):
            up = [x.copy() for x in x0]
            dn = [x.copy() for x in x0]
            up[k][idx] += eps
            dn[k][idx] -= eps
            num[idx] = (loss(up) - loss(dn)) / (2 * eps)
        numeric.append(num)
    for grads in (osc.backward(a, h, init, w), osc.chunked_backward(a, h, init, w)):
        for got, want in zip(grads, numeric):
            np.testing.assert_allclose(got, want, atol=1e-4)


def test_half_storage_accumulates_in_single_precision():
    # tests/test_networks.py:187-193: bf16 storage, float32 accumulation, within bf16's eps of
    # the exact result and closer to it than a bf16 carry
    a, b, init = problem(5, (8, 64, 256))
    a, b, init = bf16_round(a), bf16_round(b), bf16_round(init)
    exact = osc.exact(a, b, init)
    for out in (osc.sequential(a, b, init, bf16=True), osc.chunked(a, b, init, bf16=True)):
        assert np.max(np.abs(out - exact) / np.abs(exact)) <= 2.0 ** -7
    h = init.copy()
    drift = np.empty_like(a)
    for t in range(a.shape[1]):
        h = bf16_round(bf16_round(a[:, t] * h) + b[:, t])
        drift[:, t] = h
    out = osc.chunked(a, b, init, bf16=True)
    assert np.abs(out - exact).max() < np.abs(drift - exact).max()
