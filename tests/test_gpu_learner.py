"""CUDA learner parity against the CPU oracle, through the C-ABI.

Tolerances (the north star's): loss gradients within 1e-4 relative (per parameter
tensor, in the L2 norm), parameters after a full update within 1e-3 relative (on the
parameter change, per tensor), GAE targets within 1e-5; sampling bit-exact.
"""
import dataclasses

import numpy as np
import pytest
from _parity import check_grads, check_params

from boonta_b200 import configs
from boonta_b200.spec import init_params, param_layout

pytestmark = pytest.mark.gpu

GRAD_RTOL = 1e-4
PARAM_RTOL = 1e-3

# bf16 tensor-core operands: gradients and parameters are checked against the oracle's
# bf16-operand arithmetic evaluated in float64, with bounds calibrated by the float32 oracle's
# own distance from it (tests/_parity.py gives the reasoning). The targets and statistics below
# get bf16 bounds: the probability ratios of two bf16 implementations differ by ~1e-3, so a
# sample whose ratio lies that close to 1 +- clip_coefficient can fall on either side; the
# clip fraction (a count over the minibatch) gets an absolute bound of 1 % of the rows.
BF16_TOL = {"target_rtol": 1e-2, "target_atol": 3e-3, "stats_rtol": 1e-2, "stats_atol": 2e-3,
            "clipfrac_atol": 1e-2}
FP32_TOL = {"grad": GRAD_RTOL, "param": PARAM_RTOL, "params": PARAM_RTOL, "target_rtol": 1e-4,
            "target_atol": 1e-4, "stats_rtol": 2e-3, "stats_atol": 2e-4}


def tolerances(w):
    return BF16_TOL if w.precision == "bf16" else FP32_TOL


def oracle_precision(w):
    # split-bf16 (bf16x3) products carry ~16 mantissa bits: checked against plain fp32
    return "bf16" if w.precision == "bf16" else "fp32"


def small(name: str, t: int, n: int, epochs: int, minibatches: int, **kw):
    w = configs.make(name, **kw)
    return w.scaled(num_steps=t, num_envs=n, num_minibatches=minibatches, update_epochs=epochs)


def normalized(w):
    """The same workload with normalize_advantage=True (boonta/algorithms/ppo.py:220-221)."""
    return dataclasses.replace(w, ppo=dataclasses.replace(w.ppo, normalize_advantage=True))


CASES = {
    "c1": lambda: configs.c1(),  # full size: CPU-runnable reference case
    "c2": lambda: small("c2", 8, 256, 2, 4, precision="fp32"),
    "c3": lambda: small("c3", 4, 64, 2, 2, precision="fp32"),
    "c5": lambda: small("c5", 4, 64, 2, 2, precision="fp32"),
    # bf16 tensor-core GEMMs, checked against the oracle's bf16-operand arithmetic
    "c2_bf16": lambda: small("c2", 8, 256, 2, 4, precision="bf16"),
    "c5_bf16": lambda: small("c5", 4, 128, 2, 2, precision="bf16"),
    # split-bf16 tensor-core GEMMs, checked against the plain fp32 oracle
    "c2_bf16x3": lambda: small("c2", 8, 256, 2, 4, precision="bf16x3"),
    # fp32 conv kernels handing bf16 operands to a tensor-core dense layer
    "c3_bf16x3": lambda: small("c3", 4, 64, 2, 2, precision="bf16x3"),
    "c3_bf16": lambda: small("c3", 4, 64, 2, 2, precision="bf16"),
    # advantage normalisation over the whole [T, N] batch
    "c1_norm": lambda: normalized(configs.c1()),
    "c2_bf16x3_norm": lambda: normalized(small("c2", 8, 256, 2, 4, precision="bf16x3")),
}


def _learner(w):
    from boonta_b200.learner import Learner

    return Learner.from_workload(w)


def _rel(a, b):
    return float(np.linalg.norm(np.asarray(a, np.float64) - b) / max(np.linalg.norm(b), 1e-30))


@pytest.mark.parametrize("name", list(CASES))
def test_native_layout_matches_the_python_layout(name):
    w = CASES[name]()
    lrn = _learner(w)
    native = lrn.native_layout()
    py = [(e.name, e.offset, e.shape) for e in param_layout(w.network).entries]
    assert native == py
    assert lrn.num_params == param_layout(w.network).total


@pytest.mark.parametrize("name", list(CASES))
def test_minibatch_loss_gradient_matches_the_oracle(name):
    import torch

    from boonta_b200.learner import to_device
    from oracle import ppo as oppo

    w = CASES[name]()
    lrn = _learner(w)
    params = init_params(w.network, seed=5, init=w.init)
    lrn.set_state(params)
    roll = configs.rollout(w)
    rng = np.random.default_rng(11)
    b = w.batch_size
    adv = rng.standard_normal(b).astype(np.float32)
    ret = rng.standard_normal(b).astype(np.float32)
    idx = rng.permutation(b)[: w.minibatch_size].astype(np.int32)
    dev = to_device(roll)
    g, st = lrn.loss_grads(dev, torch.as_tensor(adv, device="cuda"),
                           torch.as_tensor(ret, device="cuda"), torch.as_tensor(idx))
    torch.cuda.synchronize()
    g = lrn.layout.unflatten(g.cpu().numpy())
    mb = {
        "obs": roll["obs"].reshape(b, -1)[idx],
        "action": roll["action"].reshape(b, *roll["action"].shape[2:])[idx],
        "log_prob": roll["log_prob"].reshape(b)[idx],
        "value": roll["value"].reshape(b)[idx],
        "advantages": adv[idx],
        "returns": ret[idx],
    }
    _, ost, og32 = oppo.loss_and_grads(w.network, w.ppo, params, mb,
                                       precision=oracle_precision(w))
    tol = tolerances(w)
    if tol is BF16_TOL:
        import _cublas_ref

        _, _, og = oppo.loss_and_grads(w.network, w.ppo, params, mb,
                                       precision=oracle_precision(w), dtype=np.float64)
        hw = None
        if _cublas_ref.supported(w.network):
            _, hw = _cublas_ref.loss_and_grads(w.network, w.ppo, params, mb)
        bad = check_grads(name, w.precision, g, og, og32, hw)
        assert not bad, bad
    else:
        for k in og32:
            assert _rel(g[k], og32[k]) <= tol["grad"], (k, _rel(g[k], og32[k]))
    np.testing.assert_allclose(st.cpu().numpy(), ost, rtol=max(1e-4, tol["stats_rtol"] / 10),
                               atol=1e-6 if tol is FP32_TOL else tol["stats_atol"])


@pytest.mark.parametrize("name", list(CASES))
def test_full_update_matches_the_oracle(name):
    import torch

    from boonta_b200.learner import to_device
    from oracle import optim
    from oracle import ppo as oppo

    w = CASES[name]()
    lrn = _learner(w)
    params = init_params(w.network, seed=3, init=w.init)
    lrn.set_state(params)
    roll = configs.rollout(w)
    perms = configs.permutations(w)
    st = lrn.update(to_device(roll), torch.as_tensor(perms))
    adv, ret, boot = lrn.targets()
    torch.cuda.synchronize()
    new = lrn.params()
    op, ostate, ostats, extra = oppo.update(w.network, w.ppo, w.optimizer, params,
                                            optim.init_state(params), roll, perms,
                                            precision=oracle_precision(w))
    tol = tolerances(w)
    rt, at = tol["target_rtol"], tol["target_atol"]
    np.testing.assert_allclose(boot.cpu().numpy(), extra["bootstrap"], rtol=rt, atol=at / 10)
    np.testing.assert_allclose(adv.cpu().numpy(), extra["advantages"].ravel(), rtol=rt, atol=at)
    np.testing.assert_allclose(ret.cpu().numpy(), extra["returns"].ravel(), rtol=rt, atol=at)
    if tol is BF16_TOL:
        op64, _, _, _ = oppo.update(w.network, w.ppo, w.optimizer, params,
                                    optim.init_state(params, np.float64), roll, perms,
                                    precision=oracle_precision(w), dtype=np.float64)
        bad = check_params(name, w.precision, params, new, op64, op,
                           w.ppo.update_epochs * w.ppo.num_minibatches, w.optimizer.lr)
        assert not bad, bad
    else:
        for k in op:
            d_native = new[k].astype(np.float64) - params[k]
            d_oracle = op[k].astype(np.float64) - params[k]
            assert _rel(d_native, d_oracle) <= tol["param"], (k, _rel(d_native, d_oracle))
            assert _rel(new[k], op[k]) <= tol["params"], (k, _rel(new[k], op[k]))
    stats = st.cpu().numpy()
    clip = 3  # actor/clip_fraction (ppo.py:170-179 order)
    other = [i for i in range(stats.shape[-1]) if i != clip]
    np.testing.assert_allclose(stats[..., other], ostats[..., other], rtol=tol["stats_rtol"],
                               atol=tol["stats_atol"])
    np.testing.assert_allclose(stats[..., clip], ostats[..., clip], rtol=0,
                               atol=tol.get("clipfrac_atol", tol["stats_atol"]))
    _, _, _, count = lrn.get_state()
    assert count == w.ppo.update_epochs * w.ppo.num_minibatches


def test_update_is_deterministic():
    import torch

    from boonta_b200.learner import to_device

    w = CASES["c2"]()
    roll = to_device(configs.rollout(w))
    perms = torch.as_tensor(configs.permutations(w))
    params = init_params(w.network, seed=1)
    outs = []
    for _ in range(2):
        lrn = _learner(w)
        lrn.set_state(params)
        st = lrn.update(roll, perms)
        torch.cuda.synchronize()
        outs.append((lrn.get_state()[0].cpu().numpy(), st.cpu().numpy()))
    np.testing.assert_array_equal(outs[0][0], outs[1][0])
    np.testing.assert_array_equal(outs[0][1], outs[1][1])


def test_categorical_sampling_is_bit_exact():
    import torch

    from boonta_b200.learner import sample_categorical
    from oracle import ppo as oppo

    rng = np.random.default_rng(0)
    rows, a = 4096, 43
    logits = rng.standard_normal((rows, a)).astype(np.float32) * 3
    logits[:64, 1] = logits[:64, 0]  # exact ties between actions
    u = rng.random((rows, a), dtype=np.float32)
    u = np.clip(u, np.finfo(np.float32).tiny, None)
    for temp in (1.0, 0.5, 0.0):
        act, lp = sample_categorical(torch.as_tensor(logits, device="cuda"),
                                     torch.as_tensor(u, device="cuda"), temp)
        ea, elp = oppo.sample_categorical(logits, u, temp)
        np.testing.assert_array_equal(act.cpu().numpy(), ea)
        np.testing.assert_allclose(lp.cpu().numpy(), elp, rtol=1e-6, atol=1e-6)


@pytest.mark.parametrize("name", ["c1", "c2"])
def test_act_matches_the_oracle_forward(name):
    import torch

    from oracle import network as net
    from oracle import ppo as oppo

    w = CASES[name]()
    lrn = _learner(w)
    params = init_params(w.network, seed=2, init=w.init)
    lrn.set_state(params)
    rng = np.random.default_rng(4)
    obs = rng.standard_normal((w.num_envs, w.network.obs_dim)).astype(np.float32)
    a = w.network.action_dim
    noise = (rng.random((w.num_envs, a), dtype=np.float32) if w.network.head == "categorical"
             else rng.standard_normal((w.num_envs, a), dtype=np.float32))
    noise = np.clip(noise, 1e-6, None) if w.network.head == "categorical" else noise
    act, lp, value = lrn.act(torch.as_tensor(obs, device="cuda"), torch.as_tensor(noise, device="cuda"))
    torch.cuda.synchronize()
    out, v, _ = net.forward(w.network, params, obs)
    np.testing.assert_allclose(value.cpu().numpy(), v, rtol=1e-4, atol=1e-5)
    if w.network.head == "categorical":
        ea, elp = oppo.sample_categorical(out, noise)
        agree = (act.cpu().numpy() == ea).mean()
        assert agree > 0.99  # logits differ from the oracle's in the last bits
    else:
        sig = oppo.softplus(params["actor_head/scale"]) + 1e-3
        np.testing.assert_allclose(act.cpu().numpy(), out + sig * noise, rtol=1e-4, atol=1e-5)
