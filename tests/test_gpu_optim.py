"""The standalone clip_by_global_norm + Adam entry point (bt_clip_adam) against the oracle's
restatement of optax's update rule."""
import ctypes as C

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _opt(max_norm):
    from boonta_b200 import _lib

    return _lib.OptimizerC(3e-4, max_norm, 0.9, 0.999, 1e-8, 0.0)


@pytest.mark.parametrize("n", [1, 8191, 100003, 3_000_001])
@pytest.mark.parametrize("max_norm", [0.5, 1e6], ids=["clipped", "unclipped"])
def test_clip_adam_matches_the_oracle(n, max_norm):
    import torch

    from boonta_b200 import _lib
    from boonta_b200.spec import OptimizerConfig
    from oracle import optim

    rng = np.random.default_rng(n)
    p0 = rng.standard_normal(n).astype(np.float32)
    grads = [rng.standard_normal(n).astype(np.float32) * 0.1 for _ in range(2)]
    dev = lambda x: torch.as_tensor(x, device="cuda").contiguous()
    p, m, v = dev(p0), torch.zeros(n, device="cuda"), torch.zeros(n, device="cuda")
    opt = _opt(max_norm)
    state = optim.init_state({"w": p0})
    params = {"w": p0}
    cfg = OptimizerConfig(lr=3e-4, max_grad_norm=max_norm)
    for step, g in enumerate(grads):
        gd = dev(g)
        _lib.check(_lib.lib().bt_clip_adam(p.data_ptr(), m.data_ptr(), v.data_ptr(), gd.data_ptr(),
                                           n, step, C.byref(opt),
                                           torch.cuda.current_stream().cuda_stream))
        params, state = optim.clip_adam(params, {"w": g}, state, cfg)
    torch.cuda.synchronize()
    np.testing.assert_allclose(p.cpu().numpy(), params["w"], rtol=1e-5, atol=1e-7)
    np.testing.assert_allclose(m.cpu().numpy(), state["mu"]["w"], rtol=1e-5, atol=1e-9)
    np.testing.assert_allclose(v.cpu().numpy(), state["nu"]["w"], rtol=1e-5, atol=1e-12)


def test_clip_adam_rejects_bad_arguments():
    from boonta_b200 import _lib

    opt = _opt(0.5)
    rc = _lib.lib().bt_clip_adam(None, None, None, None, 10, 0, C.byref(opt), None)
    assert rc == _lib.BT_ERR_INVALID
