"""The update replays what its rollout acted on (the property of the reference's
tests/test_algorithms.py:297-368, "every update replays what its rollout acted on").

A rollout is collected through the act entry point (bt_learner_act, the PPO.step of
boonta/algorithms/ppo.py:57-74; bt_learner_act_recurrent for RecurrentPPO.step,
boonta/algorithms/recurrent_ppo.py:72-96), recording each step's action, log-prob and value
as the rollout's `aux`, exactly as Anakin's rollout does (boonta/podracers/anakin.py:46-76).
The learner then updates on that rollout with a zero learning rate (the reference uses
optax.sgd(0.0)), so the parameters never move and every minibatch's forward pass must
recompute the log-probs the rollout recorded. The reference asserts
max |log_prob(update) - log_prob(act)| <= 1e-5. The update exposes that gap through its
statistics: with the clip coefficient set to 1e-5, `actor/clip_fraction` counts the rows
whose probability ratio exp(lp - lp_old) leaves [1 - 1e-5, 1 + 1e-5], so it must be exactly 0,
and `actor/approximate_kl` (the mean of lp_old - lp) must be within 1e-5 of 0.
"""
import dataclasses

import numpy as np
import pytest

from boonta_b200 import configs
from boonta_b200.spec import init_params

pytestmark = pytest.mark.gpu

GAP = 1e-5


def _replay_workload(name, t, n, minibatches):
    w = configs.make(name).scaled(num_steps=t, num_envs=n, num_minibatches=minibatches,
                                  update_epochs=2)
    ppo = dataclasses.replace(w.ppo, clip_coefficient=GAP)
    opt = dataclasses.replace(w.optimizer, lr=0.0)
    return dataclasses.replace(w, ppo=ppo, optimizer=opt)


CASES = {
    "c1": lambda: _replay_workload("c1", 128, 16, 4),
    "c2_bf16x3": lambda: _replay_workload("c2", 8, 8192, 4),
    "c3": lambda: _replay_workload("c3", 8, 4096, 4),
    "c5_bf16": lambda: _replay_workload("c5", 4, 4096, 4),
}


def _noise(w, rng, n):
    a = w.network.action_dim
    if w.network.head == "categorical":
        return np.clip(rng.random((n, a), dtype=np.float32), np.finfo(np.float32).tiny, None)
    return rng.standard_normal((n, a), dtype=np.float32)


def _check(w, lrn, before, dev, perms):
    import torch

    st = lrn.update(dev, perms).cpu().numpy()
    after = lrn.get_state()[0]
    torch.cuda.synchronize()
    assert torch.equal(before, after)  # a zero learning rate moves nothing
    kl, clip = st[..., 2], st[..., 3]
    print(f"{w.name} replay: max |approximate_kl| {np.abs(kl).max():.3e}, "
          f"clip fraction max {clip.max():.3e}")
    assert np.all(clip == 0.0), clip
    assert np.abs(kl).max() <= GAP, kl


@pytest.mark.parametrize("name", list(CASES))
def test_update_replays_the_acted_log_probs(name):
    import torch

    from boonta_b200.learner import Learner, to_device

    w = CASES[name]()
    lrn = Learner.from_workload(w)
    lrn.set_state(init_params(w.network, seed=9, init=w.init))
    roll = configs.rollout(w, seed=41)
    dev = to_device(roll)
    rng = np.random.default_rng(42)
    acts, lps, vals = [], [], []
    for t in range(w.num_steps):
        noise = torch.as_tensor(_noise(w, rng, w.num_envs), device="cuda")
        a, lp, v = lrn.act(dev["obs"][t].contiguous(), noise)
        acts.append(a)
        lps.append(lp)
        vals.append(v)
    dev["action"] = torch.stack(acts).contiguous()
    dev["log_prob"] = torch.stack(lps).contiguous()
    dev["value"] = torch.stack(vals).contiguous()
    before = lrn.get_state()[0].clone()
    _check(w, lrn, before, dev, torch.as_tensor(configs.permutations(w)))


def test_recurrent_update_replays_the_acted_log_probs():
    """RecurrentPPO: the rollout is collected one step at a time from the carry the previous
    step returned (reset where first.done), its start carry and the carry entering the last
    step recorded for the update (transitions.start / the tail bootstrap)."""
    import torch

    from boonta_b200.learner import Learner, to_device

    w = _replay_workload("c4", 16, 256, 4)
    lrn = Learner.from_workload(w)
    lrn.set_state(init_params(w.network, seed=9, init=w.init))
    roll = configs.rollout(w, seed=43)
    dev = to_device(roll)
    rng = np.random.default_rng(44)
    carry = dev["carry"]
    acts, lps, vals = [], [], []
    for t in range(w.num_steps):
        if t == w.num_steps - 1:
            dev["last_carry"] = carry.contiguous()
        noise = torch.as_tensor(_noise(w, rng, w.num_envs), device="cuda")
        a, lp, v, carry = lrn.act_recurrent(dev["obs"][t].contiguous(),
                                            dev["first_done"][t].contiguous(), carry, noise)
        acts.append(a)
        lps.append(lp)
        vals.append(v)
    dev["action"] = torch.stack(acts).contiguous()
    dev["log_prob"] = torch.stack(lps).contiguous()
    dev["value"] = torch.stack(vals).contiguous()
    before = lrn.get_state()[0].clone()
    _check(w, lrn, before, dev, torch.as_tensor(configs.permutations(w)))
