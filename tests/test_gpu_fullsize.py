"""Parity at the workloads' full sizes (C2-C5 at the T x N the benchmarks run), through the
C-ABI, against the CPU oracle.

Three checks per workload, each on the precision the workload benchmarks with:

  * targets over the whole rollout: the bootstrap values V(second.obs[T-1])
    (boonta/algorithms/ppo.py:208-212; the GRU tail bootstrap of
    boonta/algorithms/recurrent_ppo.py:188-198 for C4) against the oracle's forward pass,
    and the advantages / returns against the oracle's GAE
    (boonta/algorithms/advantage_estimators.py:8-56) evaluated on the learner's own
    bootstrap values, which isolates the scan (1e-5 relative, the fp32 bound);
  * the loss gradient of one full-size minibatch (16,384 rows for C2 and C5, 65,536 for
    C3; ppo.py:148-157) per parameter tensor;
  * one full update with update_epochs = 1 (every minibatch of one epoch, with clip + Adam
    after each, ppo.py:205-233): the parameters and the logged statistics. C5's host-side
    oracle cannot hold its 8.7 GB rollout, so this check runs C5 with 256 envs (1/16 of
    the benchmark's 4,096; the network, T and the minibatch count are unchanged).

The arithmetic of the comparison is in tests/_parity.py. The yardstick is the oracle evaluated
in float64 (the same operations and operand roundings,
exact products and accurate sums). Sums over 16,384-65,536 rows in float32 carry their own
rounding, so a float32 evaluation is itself up to ~1e-4 away from that (it is printed beside
every figure as `fp32 oracle`).

Tolerances. fp32 and split-bf16 (bf16x3) arithmetic are held to the north-star bounds against
the float64 oracle: gradients 1e-4 relative per tensor (L2 norm) and parameters after the update
1e-3 relative per tensor. For a tensor that starts at zero (biases) the relative error of its
parameters is taken against the largest move Adam can make in the update (steps * lr per
element), which keeps the bound meaningful. The change each tensor made is checked as well
(an update that changed nothing fails it).

bf16 GEMM operands (C5) are compared with the oracle's bf16-operand arithmetic in float64. A
layer output that sits within float32 rounding of a bf16 rounding boundary rounds to one
neighbour in one implementation and to the other in another (one bf16 step, 2^-8 relative, in
that element), and Adam's early steps (lr * sign(g) for a fresh moment) turn a gradient element
that such flips move across zero into a full-size step in the other direction. That noise is a
property of the arithmetic, not of an implementation: a float32-accumulating evaluation of the
same bf16 arithmetic (the float32 oracle, numpy's BLAS) shows it as well. The bf16 bounds are
therefore BF16_NOISE times that float32 evaluation's own distance from the float64 oracle, with
floors of 1e-4 (gradients) and 1e-3 (parameters).
"""
import numpy as np
import pytest
from _parity import BF16_NOISE, check_grads, check_params
from _parity import rel as _rel

from boonta_b200 import configs
from boonta_b200.spec import init_params

pytestmark = pytest.mark.gpu

BOOT_RTOL = {"fp32": 1e-5, "bf16x3": 1e-5, "bf16": 1e-3}


def _oracle_precision(w):
    return "bf16" if w.precision == "bf16" else "fp32"


def _one_epoch(w):
    return w.scaled(update_epochs=1)


def _device_obs(w, seed):
    """The [T, N, D] observations made on the device with the workload's distribution."""
    import torch

    g = torch.Generator(device="cuda")
    g.manual_seed(seed)
    shape = (w.num_steps, w.num_envs, w.network.obs_dim)
    if w.obs_kind == "sparse_uniform":
        x = torch.rand(shape, generator=g, device="cuda")
        keep = torch.rand(shape, generator=g, device="cuda") >= w.obs_sparsity
        return torch.where(keep, x, torch.zeros((), device="cuda"))
    if w.obs_kind == "bernoulli":
        return (torch.rand(shape, generator=g, device="cuda") < 1 - w.obs_sparsity).float()
    return torch.randn(shape, generator=g, device="cuda")


def _rollout(w):
    """Host rollout plus its device copy. Observations too large for the host (C5) are made
    on the device only; the host dict then has no "obs" (the targets need only the
    bootstrap observation)."""
    from boonta_b200.learner import to_device

    big = w.batch_size * w.network.obs_dim > 6e8
    roll = configs.rollout(w, include_obs=not big)
    dev = to_device(roll)
    if big:
        dev["obs"] = _device_obs(w, seed=w.seed + 50)
    return roll, dev


@pytest.mark.parametrize("name", ["c2", "c3", "c4", "c5"])
def test_full_size_targets(name):
    import torch

    from boonta_b200.learner import Learner
    from oracle import gae as ogae
    from oracle import network as onet
    from oracle import recurrent as orec

    w = _one_epoch(configs.make(name))
    lrn = Learner.from_workload(w)
    params = init_params(w.network, seed=7, init=w.init)
    lrn.set_state(params)
    roll, dev = _rollout(w)
    perms = torch.as_tensor(configs.permutations(w))
    lrn.update(dev, perms, stats=False)
    adv, ret, boot = lrn.targets()
    torch.cuda.synchronize()
    adv = adv.cpu().numpy().reshape(w.num_steps, w.num_envs)
    ret = ret.cpu().numpy().reshape(w.num_steps, w.num_envs)
    boot = boot.cpu().numpy()

    if w.network.recurrent:
        seq_obs = np.stack([roll["obs"][-1], roll["bootstrap_obs"]], axis=1)
        second_done = roll["terminated"][-1] | roll["truncated"][-1]
        seq_done = np.stack([roll["first_done"][-1], second_done], axis=1)
        _, v2, _ = orec.forward_seq(w.network, params, seq_obs, seq_done, roll["last_carry"])
        oboot = v2[:, -1]
    else:
        obs_b = roll["bootstrap_obs"].astype(np.float64)
        _, oboot, _ = onet.forward(w.network, params, obs_b, _oracle_precision(w))
    rel_boot = _rel(boot, oboot)
    print(f"{w.name} bootstrap rel {rel_boot:.3e}")
    assert rel_boot <= BOOT_RTOL[w.precision], rel_boot

    # the scan itself, on the learner's own bootstrap values
    oadv, oret = ogae.gae(roll["reward"], roll["terminated"], roll["truncated"], roll["value"],
                          boot, w.ppo.gamma, w.ppo.gae_lambda)
    scale = max(1.0, float(np.abs(oadv).max()))  # the chunked scan's rounding scale
    np.testing.assert_allclose(adv, oadv, rtol=1e-5, atol=1e-6 * scale)
    np.testing.assert_allclose(ret, oret, rtol=1e-5, atol=1e-6 * scale)


def _flat_minibatch(w, rows, seed):
    """One minibatch as a flat rollout of `rows` samples (its own index space 0..rows-1), so
    that a full-size minibatch needs only its own rows on the host."""
    rng = np.random.default_rng(seed)
    d, a = w.network.obs_dim, w.network.action_dim
    obs = configs._obs(rng, w, (rows, d))
    if w.network.head == "gaussian":
        action = rng.standard_normal((rows, a), dtype=np.float32)
        lp = (-0.5 * action ** 2 - 0.5 * np.log(2 * np.pi)).sum(-1)
        lp = (lp + 0.05 * rng.standard_normal(rows)).astype(np.float32)
    else:
        action = rng.integers(0, a, rows, dtype=np.int32)
        lp = (np.log(1.0 / a) + 0.05 * rng.standard_normal(rows)).astype(np.float32)
    return {
        "obs": obs,
        "bootstrap_obs": obs[: w.num_envs] if rows >= w.num_envs else obs,
        "action": action,
        "reward": np.zeros(rows, np.float32),
        "terminated": np.zeros(rows, np.uint8),
        "truncated": np.zeros(rows, np.uint8),
        "log_prob": lp,
        "value": rng.standard_normal(rows, dtype=np.float32),
        "advantages": rng.standard_normal(rows, dtype=np.float32),
        "returns": rng.standard_normal(rows, dtype=np.float32),
    }


@pytest.mark.parametrize("name", ["c2", "c3", "c5"])
def test_full_size_minibatch_gradient(name):
    import torch

    from boonta_b200.learner import Learner, to_device
    from oracle import ppo as oppo

    w = configs.make(name)
    rows = w.minibatch_size
    lrn = Learner.from_workload(w)
    params = init_params(w.network, seed=5, init=w.init)
    lrn.set_state(params)
    mb = _flat_minibatch(w, rows, seed=31)
    idx = np.random.default_rng(32).permutation(rows).astype(np.int32)
    dev = to_device({k: v for k, v in mb.items() if k not in ("advantages", "returns")})
    g, st = lrn.loss_grads(dev, torch.as_tensor(mb["advantages"], device="cuda"),
                           torch.as_tensor(mb["returns"], device="cuda"), torch.as_tensor(idx))
    torch.cuda.synchronize()
    g = lrn.layout.unflatten(g.cpu().numpy())
    st = st.cpu().numpy()
    omb = {k: mb[k][idx] for k in ("obs", "action", "log_prob", "value", "advantages", "returns")}
    prec = _oracle_precision(w)
    _, ost, og = oppo.loss_and_grads(w.network, w.ppo, params, omb, precision=prec,
                                     dtype=np.float64)
    _, _, og32 = oppo.loss_and_grads(w.network, w.ppo, params, omb, precision=prec)
    hw = None
    if w.precision == "bf16":
        from _cublas_ref import loss_and_grads as cublas_loss_and_grads

        _, hw = cublas_loss_and_grads(w.network, w.ppo, params, omb)
    bad = check_grads(f"{w.name} rows {rows}", w.precision, g, og, og32, hw)
    assert not bad, bad
    if w.precision == "bf16":
        np.testing.assert_allclose(st, ost, rtol=1e-3, atol=2e-4)
    else:
        np.testing.assert_allclose(st, ost, rtol=1e-4, atol=1e-6)


def _update_workload(name):
    w = _one_epoch(configs.make(name))
    if name == "c5":
        # the host oracle cannot hold the full 8.7 GB C5 rollout: 256 envs (1/16)
        w = w.scaled(num_envs=256)
    return w


@pytest.mark.parametrize("name", ["c2", "c3", "c4", "c5"])
def test_full_size_update_one_epoch(name):
    import torch

    from boonta_b200.learner import Learner, to_device
    from oracle import optim
    from oracle import ppo as oppo
    from oracle import recurrent as orec

    w = _update_workload(name)
    lrn = Learner.from_workload(w)
    params = init_params(w.network, seed=3, init=w.init)
    lrn.set_state(params)
    roll = configs.rollout(w)
    perms = configs.permutations(w)
    st = lrn.update(to_device(roll), torch.as_tensor(perms))
    torch.cuda.synchronize()
    new = lrn.params()
    stats = st.cpu().numpy()

    def oracle(dtype):
        if w.network.recurrent:
            return orec.update(w.network, w.ppo, w.optimizer, params,
                               optim.init_state(params, dtype), roll, perms, dtype=dtype)
        return oppo.update(w.network, w.ppo, w.optimizer, params, optim.init_state(params, dtype),
                           roll, perms, precision=_oracle_precision(w), dtype=dtype)

    op, _, ostats, _ = oracle(np.float64)
    op32, _, ostats32, _ = oracle(np.float32)
    steps = w.ppo.update_epochs * w.ppo.num_minibatches
    bad = check_params(f"{w.name} T={w.num_steps} N={w.num_envs}", w.precision, params, new, op,
                       op32, steps, w.optimizer.lr)
    assert not bad, bad
    clip = 3  # actor/clip_fraction: a count, compared as a fraction of the rows
    other = [i for i in range(stats.shape[-1]) if i != clip]
    if w.precision == "bf16":
        # each statistic within the bf16 noise: BF16_NOISE times the float32 oracle's own
        # distance from the float64 one, plus 2e-3 (the clip fraction: 1 % of the rows). The
        # distance at one minibatch is a single draw of a trajectory's divergence (the float32
        # oracle's value mean moves 5e-4 at one minibatch and 5e-3 at another), so each
        # statistic's noise scale is its largest distance over the epoch.
        noise = np.abs(ostats32 - ostats).max(axis=(0, 1), keepdims=True)
        dev = np.abs(stats - ostats)
        allowed = BF16_NOISE * noise + 2e-3
        allowed[..., clip] = BF16_NOISE * noise[..., clip] + 1e-2
        assert np.all(dev <= allowed), (np.argwhere(dev > allowed), dev.max())
    else:
        # a sample whose probability ratio lies within the arithmetic's rounding of
        # 1 +- clip_coefficient counts on either side: up to ~16 of a minibatch's 16,384 rows
        np.testing.assert_allclose(stats[..., other], ostats[..., other], rtol=2e-3, atol=2e-4)
        np.testing.assert_allclose(stats[..., clip], ostats[..., clip], rtol=0, atol=1e-3)
