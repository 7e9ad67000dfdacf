"""PPO loss, minibatch step and full learner update (test infrastructure only).

Restates boonta/algorithms/ppo.py:76-233:
  * loss_fn (:77-146): log_prob, entropy().mean(), ratio = exp(lp - lp_old),
    approximate_kl = mean(lp_old - lp), clip_fraction = mean(|ratio - 1| > eps),
    actor_loss = -mean(min(ratio*A, clip(ratio, 1-eps, 1+eps)*A)),
    critic_loss = mean(max(0.5 (v-R)^2, 0.5 (v_old + clip(v-v_old, -eps, eps) - R)^2))
    (plain 0.5 (v-R)^2 when clip_value_loss is False), loss = actor - c_e H + c_v critic.
  * jax.value_and_grad (:155-157): the analytic gradient below follows JAX's tie rules
    for min/max (lax.min/lax.max send half of the cotangent to each operand when they
    are equal) and for clip = min(max(x, lo), hi).
  * explained variance (:167-169) with population variances; the eight logged scalars
    (:170-179) in the order STAT_NAMES.
  * update (:205-233): bootstrap value from second.obs[-1], GAE, optional advantage
    normalisation, flatten [T, N] -> [T*N] (index t*N + n), then update_epochs x
    num_minibatches steps over permutation.reshape(num_minibatches, -1).

Heads (boonta/networks/distributions.py):
  * categorical: distrax Categorical over log_softmax(logits / 1.0);
    entropy = -sum p log p (:8-38).
  * gaussian: MultivariateNormalDiag(mean, softplus(scale) + 1e-3) with a state-
    independent learned scale (the SpreadScale pattern,
    hangar/recipes/recurrent_ppo_classic_control.py:19-28; split() at :49-51).
"""
from __future__ import annotations

import numpy as np

from . import gae as gae_mod
from . import network as net
from . import optim

STAT_NAMES = (
    "actor/loss",
    "actor/entropy",
    "actor/approximate_kl",
    "actor/clip_fraction",
    "actor/advantage",
    "critic/loss",
    "critic/explained_variance",
    "critic/value",
)

LOG_2PI = float(np.log(2.0 * np.pi))


def _tie(x, m, y):
    """JAX's balanced-equality cotangent weight for x in m = min/max(x, y)."""
    return np.where(x == m, np.where(y == m, 0.5, 1.0), 0.0).astype(x.dtype)


def _clip_grad(x, lo, hi):
    """d clip(x, lo, hi) / dx with clip = minimum(maximum(x, lo), hi)."""
    u = np.maximum(x, lo)
    du = _tie(x, u, np.full_like(x, lo))
    m = np.minimum(u, hi)
    dm = _tie(u, m, np.full_like(x, hi))
    return dm * du, m


def softplus(x):
    return np.maximum(x, 0) + np.log1p(np.exp(-np.abs(x)))


def head_logprob_entropy(spec, out, action, params, dtype):
    """Per-row log-prob, per-row entropy, and the pieces needed for their gradients."""
    if spec.head == "categorical":
        z = out - out.max(-1, keepdims=True)
        lse = np.log(np.exp(z).sum(-1, keepdims=True))
        logp = z - lse
        p = np.exp(logp)
        lp = np.take_along_axis(logp, action[:, None].astype(np.int64), -1)[:, 0]
        ent = -(p * logp).sum(-1)
        return lp, ent, {"p": p, "logp": logp}
    s = params["actor_head/scale"].astype(dtype)
    sigma = (softplus(s) + dtype(1e-3)).astype(dtype)
    zed = (action - out) / sigma
    lp = (-dtype(0.5) * zed * zed - np.log(sigma) - dtype(0.5 * LOG_2PI)).sum(-1)
    ent_row = (dtype(0.5) + dtype(0.5 * LOG_2PI) + np.log(sigma)).sum()
    ent = np.full(out.shape[0], ent_row, dtype)
    return lp, ent, {"sigma": sigma, "z": zed, "s": s}


def loss_and_grads(spec, ppo, params, mb, precision="fp32", dtype=np.float32):
    """One minibatch: loss, the 8 statistics, and gradients of every parameter.
    mb: dict with obs [M, D], action, log_prob, value, advantages, returns."""
    dt = np.dtype(dtype).type
    obs = np.asarray(mb["obs"], dtype)
    m = obs.shape[0]
    out, value, cache = net.forward(spec, params, obs, precision)
    lp, ent, hc = head_logprob_entropy(spec, out, mb["action"], params, dt)
    lp_old = np.asarray(mb["log_prob"], dtype)
    adv = np.asarray(mb["advantages"], dtype)
    ret = np.asarray(mb["returns"], dtype)
    v_old = np.asarray(mb["value"], dtype)
    eps = dt(ppo.clip_coefficient)

    entropy = ent.mean()
    ratio = np.exp(lp - lp_old)
    approx_kl = (lp_old - lp).mean()
    clip_frac = (np.abs(ratio - dt(1)) > eps).astype(dtype).mean()
    dclip_r, clipped = _clip_grad(ratio, dt(1) - eps, dt(1) + eps)
    s1 = ratio * adv
    s2 = clipped * adv
    mn = np.minimum(s1, s2)
    actor_loss = -mn.mean()

    c1 = dt(0.5) * ((value - ret) ** 2)
    if ppo.clip_value_loss:
        dclip_v, cl = _clip_grad(value - v_old, -eps, eps)
        v_clipped = v_old + cl
        c2 = dt(0.5) * ((v_clipped - ret) ** 2)
        crit = np.maximum(c1, c2)
        w1, w2 = _tie(c1, crit, c2), _tie(c2, crit, c1)
        dcrit_dv = w1 * (value - ret) + w2 * (v_clipped - ret) * dclip_v
    else:
        crit = c1
        dcrit_dv = value - ret
    critic_loss = crit.mean()
    loss = actor_loss - dt(ppo.entropy_coefficient) * entropy + dt(ppo.value_coefficient) * critic_loss

    # ---- statistics (ppo.py:167-179)
    resid = ret - value
    ev = dt(1) - resid.var() / (ret.var() + dt(1e-8))
    stats = np.array(
        [actor_loss, entropy, approx_kl, clip_frac, adv.mean(), critic_loss, ev, value.mean()],
        np.float64,
    )

    # ---- gradient
    inv_m = dt(1.0 / m)
    t1, t2 = _tie(s1, mn, s2), _tie(s2, mn, s1)
    dmn_dratio = t1 * adv + t2 * adv * dclip_r
    g_lp = -(dmn_dratio * ratio) * inv_m  # dL/d lp per row
    g_ent = -dt(ppo.entropy_coefficient) * inv_m  # dL/d H_row
    d_value = dt(ppo.value_coefficient) * inv_m * dcrit_dv
    grads_extra = {}
    if spec.head == "categorical":
        p, logp = hc["p"], hc["logp"]
        onehot = np.zeros_like(p)
        onehot[np.arange(m), mb["action"].astype(np.int64)] = 1
        d_out = g_lp[:, None] * (onehot - p) + g_ent * (-p * (logp + ent[:, None]))
    else:
        sigma, zed, s = hc["sigma"], hc["z"], hc["s"]
        d_out = g_lp[:, None] * (zed / sigma)
        d_sigma = (g_lp[:, None] * ((zed * zed - dt(1)) / sigma)).sum(0) + m * g_ent / sigma
        grads_extra["actor_head/scale"] = (d_sigma * net.sigmoid(s)).astype(dtype)
    grads = net.backward(spec, params, cache, d_out.astype(dtype), d_value.astype(dtype), precision)
    grads.update(grads_extra)
    return float(loss), stats, grads


def update(spec, ppo, opt, params, opt_state, rollout, perms, precision="fp32",
           dtype=np.float32, max_minibatches=None):
    """The full learner step of one device. Returns (params, opt_state, stats [E, M, 8],
    extras). `perms` is [E, T*N]; `max_minibatches` truncates the run (CPU timing only)."""
    t, n = rollout["reward"].shape
    b = t * n
    obs_b = np.asarray(rollout["bootstrap_obs"], dtype)
    _, boot, _ = net.forward(spec, params, obs_b, precision)
    adv, ret = gae_mod.gae(
        rollout["reward"], rollout["terminated"], rollout["truncated"], rollout["value"],
        boot, ppo.gamma, ppo.gae_lambda, dtype=dtype,
    )
    if ppo.normalize_advantage:
        adv = (adv - adv.mean()) / (adv.std() + np.dtype(dtype).type(1e-8))
    flat = {
        "obs": rollout["obs"].reshape(b, -1),
        "action": rollout["action"].reshape(b, *rollout["action"].shape[2:]),
        "log_prob": rollout["log_prob"].reshape(b),
        "value": rollout["value"].reshape(b),
        "advantages": adv.reshape(b),
        "returns": ret.reshape(b),
    }
    mbs = ppo.num_minibatches
    stats = np.zeros((ppo.update_epochs, mbs, 8))
    done = 0
    for e in range(ppo.update_epochs):
        idx = np.asarray(perms[e]).reshape(mbs, -1)
        for k in range(mbs):
            if max_minibatches is not None and done >= max_minibatches:
                return params, opt_state, stats, {"advantages": adv, "returns": ret, "bootstrap": boot}
            mb = {key: val[idx[k]] for key, val in flat.items()}
            _, st, grads = loss_and_grads(spec, ppo, params, mb, precision, dtype)
            params, opt_state = optim.clip_adam(params, grads, opt_state, opt, dtype)
            stats[e, k] = st
            done += 1
    return params, opt_state, stats, {"advantages": adv, "returns": ret, "bootstrap": boot}


def sample_categorical(logits, uniforms, temperature=1.0):
    """Categorical._sample_n (boonta/networks/distributions.py:9-23): argmax over
    log_softmax(logits / temperature) + gumbel, gumbel = -log(-log(u)); temperature 0 is the
    greedy argmax with log-prob 0. The gumbel noise and the log_softmax are evaluated in
    double and rounded once to float32, then added in float32 (first index wins ties)."""
    logits = np.asarray(logits, np.float32)
    if not temperature > 0:
        return logits.argmax(-1).astype(np.int32), np.zeros(logits.shape[0], np.float32)
    cooled = (logits / np.float32(temperature)).astype(np.float64)
    mx = cooled.max(-1, keepdims=True)
    lse = np.log(np.exp(cooled - mx).sum(-1, keepdims=True)) + mx
    lsm = cooled - lse
    v = lsm.astype(np.float32)
    if uniforms is not None:
        g = (-np.log(-np.log(np.asarray(uniforms, np.float32).astype(np.float64)))).astype(np.float32)
        v = (v + g).astype(np.float32)
    action = v.argmax(-1).astype(np.int32)
    lp = np.take_along_axis(lsm, action[:, None].astype(np.int64), -1)[:, 0].astype(np.float32)
    return action, lp
