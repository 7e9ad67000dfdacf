"""The boonta-compatible PPO / RecurrentPPO classes (boonta/algorithms/ppo.py:17-233,
recurrent_ppo.py:18-281): construction rules on CPU; init/step/update against the oracle
on the GPU."""
import numpy as np
import pytest

from boonta_b200 import configs
from boonta_b200.ppo import PPO, RecurrentPPO, Timestep, Transition, generalized_advantage_estimator
from boonta_b200.spec import OptimizerConfig, param_layout


def test_constructor_rejects_what_the_learner_does_not_implement():
    w = configs.c1()
    with pytest.raises(NotImplementedError):
        PPO(w.ppo, w.network, w.optimizer, auxiliary_losses=(lambda *a: 0.0,))
    with pytest.raises(NotImplementedError):
        PPO(w.ppo, w.network, w.optimizer, advantage_estimator=lambda *a: None)
    with pytest.raises(NotImplementedError):
        PPO(w.ppo, object(), w.optimizer)
    with pytest.raises(NotImplementedError):
        PPO(w.ppo, w.network, object())
    with pytest.raises(NotImplementedError):
        PPO(w.ppo, configs.c4().network, w.optimizer)  # GRU torso -> RecurrentPPO
    with pytest.raises(NotImplementedError):
        RecurrentPPO(w.ppo, w.network, w.optimizer)
    ppo = PPO(w.ppo, w.network, w.optimizer)
    assert ppo.cfg is w.ppo and isinstance(ppo.optimizer, OptimizerConfig)


def _transition(w, roll, dev):
    import torch

    t = {k: torch.as_tensor(v).to(dev) for k, v in roll.items()}
    obs = t["obs"]
    second_obs = torch.cat([obs[1:], t["bootstrap_obs"][None]], 0)
    first = Timestep(obs=obs, terminated=torch.zeros_like(t["terminated"]),
                     truncated=torch.zeros_like(t["truncated"]))
    if "first_done" in t:
        first = Timestep(obs=obs, terminated=t["first_done"], truncated=torch.zeros_like(t["truncated"]))
    second = Timestep(obs=second_obs, action=t["action"], reward=t["reward"],
                      terminated=t["terminated"], truncated=t["truncated"])
    carry = None
    if "carry" in t:
        carry = torch.stack([t["carry"]] + [t["carry"]] * (w.num_steps - 2) + [t["last_carry"]])
    return Transition(first=first, second=second,
                      aux={"log_prob": t["log_prob"], "value": t["value"]}, carry=carry)


@pytest.mark.gpu
def test_ppo_update_matches_the_learner_and_the_oracle():
    import torch

    from boonta_b200.learner import Learner, to_device
    from oracle import optim
    from oracle import ppo as oppo

    w = configs.make("c2", precision="fp32").scaled(num_steps=8, num_envs=128,
                                                    num_minibatches=4, update_epochs=2)
    ppo = PPO(w.ppo, w.network, w.optimizer)
    roll = configs.rollout(w, seed=2)
    tr = _transition(w, roll, "cuda")
    state, carry = ppo.init(7, Timestep(obs=tr.first.obs[0]))
    assert carry is None and int(state.step) == 0 and state.optimizer_state.count == 0
    params0 = state.params.cpu().numpy().copy()
    new = ppo.update(state, 3, tr)
    assert int(new.step) == 0  # ppo.py:193-197 leaves step to the podracer
    assert new.optimizer_state.count == w.ppo.update_epochs * w.ppo.num_minibatches
    # the same permutations through the learner directly
    perms = ppo._permutations(3, w.num_steps * w.num_envs, "cuda")
    lrn = Learner.from_workload(w)
    lrn.set_state(params0)
    lrn.update(to_device(roll), perms)
    np.testing.assert_array_equal(new.params.cpu().numpy(), lrn.get_state()[0].cpu().numpy())
    # and the oracle: parameter change within 1e-3 relative per tensor
    layout = param_layout(w.network)
    p0 = layout.unflatten(params0)
    op, _, _, _ = oppo.update(w.network, w.ppo, w.optimizer, p0, optim.init_state(p0), roll,
                              perms.cpu().numpy())
    got = layout.unflatten(new.params.cpu().numpy())
    for k in op:
        d_native = np.asarray(got[k], np.float64) - p0[k]
        d_oracle = np.asarray(op[k], np.float64) - p0[k]
        err = np.linalg.norm(d_native - d_oracle) / max(np.linalg.norm(d_oracle), 1e-30)
        assert err <= 1e-3, (k, err)
    # the state passes through again (learner reloads only when the state changes)
    again = ppo.update(new, 4, tr)
    assert again.optimizer_state.count == 2 * w.ppo.update_epochs * w.ppo.num_minibatches


@pytest.mark.gpu
def test_ppo_step_samples_with_the_learner_act():
    import torch

    w = configs.c1()
    ppo = PPO(w.ppo, w.network, w.optimizer, init_scheme="orthogonal")
    obs = torch.randn(w.num_envs, w.network.obs_dim, device="cuda")
    state, carry = ppo.init(0, Timestep(obs=obs))
    s2, c2, action, aux = ppo.step(state, carry, 5, Timestep(obs=obs))
    assert s2 is state and c2 is None
    assert action.shape == (w.num_envs,) and action.dtype == torch.int32
    assert aux["log_prob"].shape == (w.num_envs,) and aux["value"].shape == (w.num_envs,)
    assert bool((aux["log_prob"] <= 0).all())
    _, _, action2, _ = ppo.step(state, carry, 5, Timestep(obs=obs))
    assert torch.equal(action, action2)  # same key, same draws


@pytest.mark.gpu
def test_gae_estimator_matches_the_oracle():
    import torch

    from oracle import gae as ogae

    rng = np.random.default_rng(0)
    t, n = 16, 32
    r = rng.standard_normal((t, n)).astype(np.float32)
    term = (rng.random((t, n)) < 0.1).astype(np.uint8)
    trunc = (rng.random((t, n)) < 0.05).astype(np.uint8)
    v = rng.standard_normal((t, n)).astype(np.float32)
    boot = rng.standard_normal(n).astype(np.float32)
    c = lambda x: torch.as_tensor(x).cuda()
    tr = Transition(second=Timestep(obs=None, reward=c(r), terminated=c(term), truncated=c(trunc)))
    adv, ret = generalized_advantage_estimator(tr, c(v), c(boot), 0.99, 0.95)
    ra, rr = ogae.gae(r, term, trunc, v, boot, 0.99, 0.95)
    scale = max(1.0, float(np.abs(ra).max()))
    np.testing.assert_allclose(adv.cpu().numpy(), ra, rtol=1e-5, atol=1e-6 * scale)
    np.testing.assert_allclose(ret.cpu().numpy(), rr, rtol=1e-5, atol=1e-6 * scale)


@pytest.mark.gpu
def test_recurrent_ppo_update_runs_and_counts():
    import torch

    w = configs.make("c4").scaled(num_steps=8, num_envs=32, num_minibatches=2, update_epochs=2)
    ppo = RecurrentPPO(w.ppo, w.network, w.optimizer)
    roll = configs.rollout(w, seed=1)
    tr = _transition(w, roll, "cuda")
    state, carry = ppo.init(1, Timestep(obs=tr.first.obs[0], reward=tr.second.reward[0]))
    assert tuple(carry.shape) == (w.num_envs, w.network.torso[-1].features)
    new = ppo.update(state, 2, tr)
    assert new.optimizer_state.count == w.ppo.update_epochs * w.ppo.num_minibatches
    assert bool(np.isfinite(new.params.cpu().numpy()).all())
    # act with the carry (RecurrentPPO.step): the carry changes, a reset zeroes it first
    obs = tr.first.obs[0]
    done = torch.zeros(w.num_envs, dtype=torch.bool, device="cuda")
    s2, c2, action, aux = ppo.step(new, carry, 3, Timestep(obs=obs, terminated=done))
    assert s2 is new and tuple(c2.shape) == tuple(carry.shape)
    assert action.shape == (w.num_envs,) and aux["value"].shape == (w.num_envs,)
    assert bool((aux["log_prob"] <= 0).all()) and not torch.equal(c2, carry)
    _, c3, _, _ = ppo.step(new, c2, 3, Timestep(obs=obs, terminated=~done))
    _, c4, _, _ = ppo.step(new, torch.zeros_like(c2), 3, Timestep(obs=obs))
    assert torch.equal(c3, c4)  # reset everywhere == starting from a zero carry
