"""The oracle's analytic loss gradient against central finite differences in float64,
for every network family of the five workloads (tiny widths)."""
import numpy as np
import pytest

from boonta_b200.spec import Conv3x3, Dense, NetworkSpec, PPOConfig, init_params
from oracle import ppo as oppo

PPO = PPOConfig(num_minibatches=1, update_epochs=1, clip_coefficient=0.2, clip_value_loss=True,
                entropy_coefficient=0.01, value_coefficient=0.5, gamma=0.99, gae_lambda=0.95)

NETS = {
    "c1_mlp_tanh": NetworkSpec(4, (Dense(8, "tanh"), Dense(8, "tanh")), head="categorical", action_dim=2),
    "c2_separate_silu_gaussian": NetworkSpec(
        5, (Dense(8, "silu"), Dense(8, "silu")), critic=(Dense(6, "silu"), Dense(6, "silu")),
        head="gaussian", action_dim=3),
    "c3_conv": NetworkSpec(4 * 4 * 2, (Conv3x3(3, 4, 4, 2, "relu"), Dense(8, "relu")),
                           head="categorical", action_dim=4),
    "c5_layernorm": NetworkSpec(7, (Dense(8, "relu", layernorm=True), Dense(8, "relu", layernorm=True)),
                                head="categorical", action_dim=5),
}


def minibatch(spec, rows, rng):
    mb = {"obs": rng.standard_normal((rows, spec.obs_dim))}
    if spec.head == "gaussian":
        mb["action"] = rng.standard_normal((rows, spec.action_dim))
    else:
        mb["action"] = rng.integers(0, spec.action_dim, rows)
    mb["log_prob"] = rng.standard_normal(rows) * 0.3 - 1.0
    mb["value"] = rng.standard_normal(rows)
    mb["advantages"] = rng.standard_normal(rows)
    mb["returns"] = rng.standard_normal(rows)
    return mb


@pytest.mark.parametrize("name", list(NETS))
def test_analytic_gradient_matches_finite_differences(name):
    spec = NETS[name]
    rng = np.random.default_rng(7)
    params = {k: v.astype(np.float64) for k, v in init_params(spec, seed=1).items()}
    # give biases, LN parameters and the gaussian scale non-trivial values
    for k in params:
        params[k] = params[k] + 0.1 * rng.standard_normal(params[k].shape)
    mb = minibatch(spec, 12, rng)
    loss, _, grads = oppo.loss_and_grads(spec, PPO, params, mb, dtype=np.float64)
    h = 1e-6
    checked = 0
    for k, p in params.items():
        flat = p.ravel()
        for i in rng.choice(flat.size, size=min(6, flat.size), replace=False):
            orig = flat[i]
            flat[i] = orig + h
            lp, _, _ = oppo.loss_and_grads(spec, PPO, params, mb, dtype=np.float64)
            flat[i] = orig - h
            lm, _, _ = oppo.loss_and_grads(spec, PPO, params, mb, dtype=np.float64)
            flat[i] = orig
            fd = (lp - lm) / (2 * h)
            an = grads[k].ravel()[i]
            assert abs(fd - an) <= 1e-6 + 1e-4 * abs(fd), (k, i, fd, an)
            checked += 1
    assert checked > 10


def test_statistics_follow_the_reference_definitions():
    spec = NETS["c1_mlp_tanh"]
    rng = np.random.default_rng(0)
    params = init_params(spec, seed=0)
    mb = minibatch(spec, 64, rng)
    mb = {k: (v.astype(np.float32) if v.dtype == np.float64 else v) for k, v in mb.items()}
    loss, stats, _ = oppo.loss_and_grads(spec, PPO, params, mb)
    from oracle import network as net

    out, value, _ = net.forward(spec, params, mb["obs"])
    ev = 1 - np.var(mb["returns"] - value) / (np.var(mb["returns"]) + 1e-8)
    assert stats[6] == pytest.approx(ev, rel=1e-5)
    assert stats[7] == pytest.approx(value.mean(), rel=1e-5, abs=1e-7)
    assert stats[4] == pytest.approx(mb["advantages"].mean(), rel=1e-6)


def test_recurrent_bptt_gradient_matches_finite_differences():
    """GRU torso (rnn.py:30-54 + flax GRUCell) with resets: analytic BPTT vs central
    differences in float64."""
    from boonta_b200.spec import GRU
    from oracle import recurrent

    spec = NetworkSpec(5, (Dense(6, "relu"), GRU(4)), head="categorical", action_dim=3)
    rng = np.random.default_rng(3)
    params = {k: v.astype(np.float64) + 0.1 * rng.standard_normal(v.shape)
              for k, v in init_params(spec, seed=2).items()}
    b, t = 3, 5
    traj = {
        "obs": rng.standard_normal((b, t, 5)),
        "done": (rng.random((b, t)) < 0.3).astype(np.uint8),
        "action": rng.integers(0, 3, (b, t)),
        "log_prob": rng.standard_normal((b, t)) * 0.3 - 1.0,
        "value": rng.standard_normal((b, t)),
        "advantages": rng.standard_normal((b, t)),
        "returns": rng.standard_normal((b, t)),
    }
    carry = rng.standard_normal((b, 4)) * 0.5
    _, _, grads = recurrent.loss_and_grads(spec, PPO, params, traj, carry, dtype=np.float64)
    h = 1e-6
    for k, p in params.items():
        flat = p.ravel()
        for i in rng.choice(flat.size, size=min(5, flat.size), replace=False):
            orig = flat[i]
            flat[i] = orig + h
            lp, _, _ = recurrent.loss_and_grads(spec, PPO, params, traj, carry, dtype=np.float64)
            flat[i] = orig - h
            lm, _, _ = recurrent.loss_and_grads(spec, PPO, params, traj, carry, dtype=np.float64)
            flat[i] = orig
            fd = (lp - lm) / (2 * h)
            an = grads[k].ravel()[i]
            assert abs(fd - an) <= 1e-6 + 1e-4 * abs(fd), (k, i, fd, an)
