"""The native linear scan (bt_linear_scan / bt_linear_scan_backward, boonta_b200.scan) against
the oracle (oracle/scan.py): bit-identical to the oracle's restatement of the kernels' chunked
order, within the reference's tolerances (tests/test_networks.py:141-210) of its sequential
order, for float32 and bfloat16 storage, ragged widths and step counts, both init dtypes."""
import numpy as np
import pytest

from oracle import scan as osc
from oracle.network import bf16_round

pytestmark = pytest.mark.gpu

SHAPES = [(4, 16, 128), (2, 8, 100), (3, 1, 33), (1, 67, 64), (2, 200, 40), (5, 128, 256),
          (8, 64, 256)]


def problem(seed, shape):
    rng = np.random.default_rng(seed)
    a = (rng.uniform(size=shape) * 0.9 + 0.05).astype(np.float32)
    b = rng.uniform(size=shape).astype(np.float32)
    init = rng.standard_normal((shape[0], shape[2])).astype(np.float32)
    cot = rng.standard_normal(shape).astype(np.float32)
    return a, b, init, cot


def _t(x, dtype):
    import torch

    return torch.tensor(x, device="cuda").to(dtype)


def _np(t):
    import torch

    t = t.detach()
    return t.float().cpu().numpy() if t.dtype == torch.bfloat16 else t.cpu().numpy()


@pytest.mark.parametrize("shape", SHAPES, ids=lambda s: "x".join(map(str, s)))
@pytest.mark.parametrize("half,init_half", [(False, False), (True, False), (True, True),
                                            (False, True)])
def test_scan_and_its_gradient_match_the_oracle(shape, half, init_half):
    import torch

    from boonta_b200.scan import scan

    a, b, init, cot = problem(sum(shape), shape)
    if half:
        a, b, cot = bf16_round(a), bf16_round(b), bf16_round(cot)
    if init_half:
        init = bf16_round(init)
    dt = torch.bfloat16 if half else torch.float32
    ta, tb = _t(a, dt).requires_grad_(), _t(b, dt).requires_grad_()
    ti = _t(init, torch.bfloat16 if init_half else torch.float32).requires_grad_()
    h = scan(ta, tb, ti)
    assert h.dtype == dt
    h.backward(_t(cot, dt))
    torch.cuda.synchronize()
    got = _np(h)
    np.testing.assert_array_equal(got, osc.chunked(a, b, init, bf16=half))
    da, db, dinit = osc.chunked_backward(a, got, init, cot, bf16=half)
    np.testing.assert_array_equal(_np(ta.grad), da)
    np.testing.assert_array_equal(_np(tb.grad), db)
    np.testing.assert_array_equal(_np(ti.grad), bf16_round(dinit) if init_half else dinit)
    # the reference's sequential order
    seq = osc.sequential(a, b, init, bf16=half)
    if half:
        np.testing.assert_allclose(got, seq, rtol=2 ** -7, atol=1e-6)
    else:
        np.testing.assert_allclose(got, seq, rtol=1e-5, atol=1e-5)
        sda, sdb, sdi = osc.backward(a, seq, init, cot)
        for g, w in ((ta.grad, sda), (tb.grad, sdb)):
            np.testing.assert_allclose(_np(g), w, rtol=1e-4, atol=1e-4)
        # dinit is stored in init's dtype
        np.testing.assert_allclose(_np(ti.grad), sdi, rtol=2 ** -8 if init_half else 1e-4,
                                   atol=1e-4)


def test_extra_feature_axes_are_folded_like_the_reference():
    import torch

    from boonta_b200.scan import scan, sequential

    rng = np.random.default_rng(9)
    a = torch.tensor(rng.uniform(0.1, 0.9, (2, 12, 3, 32)), dtype=torch.float32, device="cuda")
    b = torch.tensor(rng.uniform(size=(2, 12, 3, 32)), dtype=torch.float32, device="cuda")
    init = torch.tensor(rng.standard_normal((2, 3, 32)), dtype=torch.float32, device="cuda")
    out = scan(a, b, init)
    fold = lambda x: torch.movedim(x, 1, -2).reshape(-1, 12, 32)
    want = torch.movedim(sequential(fold(a), fold(b), init.reshape(-1, 32)).reshape(2, 3, 12, 32), -2, 1)
    torch.testing.assert_close(out, want, rtol=1e-5, atol=1e-5)


def test_empty_shapes_and_bad_arguments():
    import torch

    from boonta_b200 import _lib
    from boonta_b200.scan import scan

    z = torch.zeros((0, 4, 8), device="cuda")
    assert scan(z, z, torch.zeros((0, 8), device="cuda")).shape == (0, 4, 8)
    with pytest.raises(RuntimeError, match="dtype"):
        _lib.check(_lib.lib().bt_linear_scan(None, None, None, None, 1, 1, 1, 7, 0, None))
    with pytest.raises(RuntimeError, match="null"):
        _lib.check(_lib.lib().bt_linear_scan(None, None, None, None, 1, 1, 1, 0, 0, None))
