"""RecurrentPPO learner (GRU torso, C4 workload) against the recurrent oracle through the
C-ABI: full update with env-minibatches, resets and the tail bootstrap. fp32 throughout;
tolerances as for the fp32 feed-forward learner (params within 1e-3 after a full update)."""
import numpy as np
import pytest

from boonta_b200 import configs
from boonta_b200.spec import init_params, param_layout

pytestmark = pytest.mark.gpu


def _rel(a, b):
    return float(np.linalg.norm(np.asarray(a, np.float64) - b) / max(np.linalg.norm(b), 1e-30))


def small_c4(t=16, n=64, epochs=2, minibatches=4):
    return configs.c4().scaled(num_steps=t, num_envs=n, num_minibatches=minibatches,
                               update_epochs=epochs)


def test_recurrent_layout_matches_the_python_layout():
    from boonta_b200.learner import Learner

    w = small_c4()
    lrn = Learner.from_workload(w)
    py = [(e.name, e.offset, e.shape) for e in param_layout(w.network).entries]
    assert lrn.native_layout() == py


@pytest.mark.parametrize("shape", [(16, 64, 2, 4), (9, 24, 1, 3)], ids=["t16n64", "t9n24"])
def test_recurrent_update_matches_the_oracle(shape):
    import torch

    from boonta_b200.learner import Learner, to_device
    from oracle import optim, recurrent

    w = small_c4(*shape)
    lrn = Learner.from_workload(w)
    params = init_params(w.network, seed=3)
    lrn.set_state(params)
    roll = configs.rollout(w)
    perms = configs.permutations(w)
    st = lrn.update(to_device(roll), torch.as_tensor(perms))
    adv, ret, boot = lrn.targets()
    torch.cuda.synchronize()
    new = lrn.params()
    op, _, ostats, extra = recurrent.update(w.network, w.ppo, w.optimizer, params,
                                            optim.init_state(params), roll, perms)
    np.testing.assert_allclose(boot.cpu().numpy(), extra["bootstrap"], rtol=1e-4, atol=1e-5)
    np.testing.assert_allclose(adv.cpu().numpy(), extra["advantages"].ravel(), rtol=1e-4, atol=1e-4)
    np.testing.assert_allclose(ret.cpu().numpy(), extra["returns"].ravel(), rtol=1e-4, atol=1e-4)
    for k in op:
        assert _rel(new[k], op[k]) <= 1e-3, (k, _rel(new[k], op[k]))
        d_native = new[k].astype(np.float64) - params[k]
        d_oracle = op[k].astype(np.float64) - params[k]
        assert _rel(d_native, d_oracle) <= 1e-3, (k, _rel(d_native, d_oracle))
    np.testing.assert_allclose(st.cpu().numpy(), ostats, rtol=2e-3, atol=2e-4)


@pytest.mark.parametrize("n", [64, 16], ids=["n64", "n16"])
def test_recurrent_act_matches_the_oracle(n):
    """bt_learner_act_recurrent (RecurrentPPO.step): value, carry out and the sample against
    the oracle's forward over a one-step sequence from the same carry and resets, then a
    second step chained on the returned carry."""
    import torch

    from boonta_b200.learner import Learner
    from oracle import ppo as oppo
    from oracle import recurrent

    w = small_c4(t=16, n=n, epochs=1, minibatches=2)
    lrn = Learner.from_workload(w)
    params = init_params(w.network, seed=5)
    lrn.set_state(params)
    rng = np.random.default_rng(11)
    h, a, d = w.network.torso[-1].features, w.network.action_dim, w.network.obs_dim
    obs = rng.standard_normal((2, n, d)).astype(np.float32)
    carry = (0.1 * rng.standard_normal((n, h))).astype(np.float32)
    reset = np.stack([(rng.random(n) < 0.3), np.zeros(n, bool)]).astype(np.uint8)
    u = rng.random((2, n, a)).astype(np.float32).clip(np.finfo(np.float32).tiny, None)
    c = lambda x: torch.as_tensor(x).cuda()
    out, val, cache = recurrent.forward_seq(w.network, params, obs.transpose(1, 0, 2),
                                            reset.T, carry)
    cur = c(carry)
    for t in range(2):
        action, lp, value, cur = lrn.act_recurrent(c(obs[t]), c(reset[t]), cur, c(u[t]))
        torch.cuda.synchronize()
        np.testing.assert_allclose(value.cpu().numpy(), val[:, t], rtol=1e-4, atol=1e-5)
        np.testing.assert_allclose(cur.cpu().numpy(), cache["hs"][:, t], rtol=1e-4, atol=1e-5)
        ref_action, ref_lp = oppo.sample_categorical(out[:, t], u[t])
        np.testing.assert_array_equal(action.cpu().numpy(), ref_action)
        np.testing.assert_allclose(lp.cpu().numpy(), ref_lp, rtol=1e-4, atol=1e-5)
