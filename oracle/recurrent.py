"""RecurrentPPO.update with a GRU torso (test infrastructure only).

Restates boonta/algorithms/recurrent_ppo.py:98-281 with the network of the C4 workload
(hangar/recipes/recurrent_ppo_minatar.py with the linear encoder: obs -> Dense + ReLU ->
RNN(GRUCell) -> heads), and boonta/networks/blocks/rnn.py:11-59:

  * the carry is reset to the cell's initial carry (zeros) before step t wherever
    first.done[t] (rnn.py:42-45, reset_carry :11-16);
  * tail bootstrap (recurrent_ppo.py:188-198): a 2-step sequence (first[-1], second[-1])
    from the carry entering step T-1, value of the second step;
  * minibatches over envs (recurrent_ppo.py:269-276), each a full [mb_envs, T] sequence
    from transitions.start (the carry entering step 0), losses averaged over mb_envs*T.

flax.linen.GRUCell (flax 0.12.8, not vendored) is restated from its documented math:
  r = sigmoid(x W_ir + b_ir + h W_hr)          z = sigmoid(x W_iz + b_iz + h W_hz)
  n = tanh(x W_in + b_in + r * (h W_hn + b_hn))   h' = (1 - z) * n + z * h
with the input kernels stored as one [K, 3H] matrix (r | z | n) plus bias [3H], the
recurrent kernels as [H, 3H] and b_hn as [H]. Parity against flax itself is unpinned.
"""
from __future__ import annotations

import numpy as np

from . import gae as gae_mod
from . import network as net
from . import optim
from .ppo import _clip_grad, _tie, head_logprob_entropy


def _sig(x):
    return 1.0 / (1.0 + np.exp(-x))


def gru_layer_names(spec):
    return [i for i, layer in enumerate(spec.torso) if type(layer).__name__ == "GRU"]


def forward_seq(spec, params, obs, done, carry, dtype=np.float32):
    """obs [B, T, D], done [B, T] (reset before step t), carry [B, H].
    Returns (out [B, T, A], value [B, T], cache)."""
    dt = np.dtype(dtype).type
    b, t, _ = obs.shape
    x = obs.astype(dtype)
    cache = {"layers": []}
    h_in = x
    gru_idx = None
    for i, layer in enumerate(spec.torso):
        p = f"torso/{i}"
        if type(layer).__name__ == "GRU":
            gru_idx = i
            break
        z = h_in @ params[f"{p}/kernel"].astype(dtype) + params[f"{p}/bias"].astype(dtype)
        h = net.activation(z, layer.activation)
        cache["layers"].append({"x": h_in, "z": z, "h": h, "layer": layer, "prefix": p})
        h_in = h
    assert gru_idx == len(spec.torso) - 1, "the GRU must be the last torso layer"
    p = f"torso/{gru_idx}"
    wi = params[f"{p}/input_kernel"].astype(dtype)
    bi = params[f"{p}/input_bias"].astype(dtype)
    wh = params[f"{p}/recurrent_kernel"].astype(dtype)
    bhn = params[f"{p}/hn_bias"].astype(dtype)
    hdim = wh.shape[0]
    xp = h_in @ wi + bi  # [B, T, 3H]
    hs = np.zeros((b, t, hdim), dtype)
    saved = {k: np.zeros((b, t, hdim), dtype) for k in ("hin", "r", "z", "n", "hpn")}
    h = carry.astype(dtype)
    for s in range(t):
        h = np.where(done[:, s, None].astype(bool), dt(0), h)
        hp = h @ wh
        r = _sig(xp[:, s, :hdim] + hp[:, :hdim])
        zg = _sig(xp[:, s, hdim:2 * hdim] + hp[:, hdim:2 * hdim])
        hpn = hp[:, 2 * hdim:] + bhn
        n = np.tanh(xp[:, s, 2 * hdim:] + r * hpn)
        new = (dt(1) - zg) * n + zg * h
        for k, v in (("hin", h), ("r", r), ("z", zg), ("n", n), ("hpn", hpn)):
            saved[k][:, s] = v
        hs[:, s] = new
        h = new
    cache.update(gru_in=h_in, saved=saved, hs=hs, prefix=p, hdim=hdim)
    out = hs @ params["actor_head/kernel"].astype(dtype) + params["actor_head/bias"].astype(dtype)
    value = (hs @ params["critic_head/kernel"].astype(dtype) + params["critic_head/bias"].astype(dtype))[..., 0]
    return out, value, cache


def backward_seq(spec, params, cache, d_out, d_value, done, dtype=np.float32):
    """Gradients of all parameters given dL/d out [B, T, A] and dL/d value [B, T] (BPTT)."""
    dt = np.dtype(dtype).type
    hs = cache["hs"]
    grads = {}
    flat = lambda a: a.reshape(-1, a.shape[-1])
    grads["actor_head/kernel"] = flat(hs).T @ flat(d_out)
    grads["actor_head/bias"] = flat(d_out).sum(0)
    dv = d_value[..., None]
    grads["critic_head/kernel"] = flat(hs).T @ flat(dv)
    grads["critic_head/bias"] = flat(dv).sum(0)
    d_hs = d_out @ params["actor_head/kernel"].astype(dtype).T + dv @ params["critic_head/kernel"].astype(dtype).T
    p, hdim = cache["prefix"], cache["hdim"]
    wh = params[f"{p}/recurrent_kernel"].astype(dtype)
    wi = params[f"{p}/input_kernel"].astype(dtype)
    sv = cache["saved"]
    b, t, _ = hs.shape
    dxp = np.zeros((b, t, 3 * hdim), dtype)
    dhp = np.zeros((b, t, 3 * hdim), dtype)
    carry_grad = np.zeros((b, hdim), dtype)
    for s in reversed(range(t)):
        dh = d_hs[:, s] + carry_grad
        r, zg, n, hpn, hin = (sv[k][:, s] for k in ("r", "z", "n", "hpn", "hin"))
        dn = dh * (dt(1) - zg)
        dz = dh * (hin - n)
        dhin = dh * zg
        dan = dn * (dt(1) - n * n)
        dr = dan * hpn
        dar = dr * r * (dt(1) - r)
        daz = dz * zg * (dt(1) - zg)
        dxp[:, s] = np.concatenate([dar, daz, dan], -1)
        dhp[:, s] = np.concatenate([dar, daz, dan * r], -1)
        dhin = dhin + dhp[:, s] @ wh.T
        # the reset before step s cut the dependence on the previous step's output
        carry_grad = np.where(done[:, s, None].astype(bool), dt(0), dhin)
    grads[f"{p}/recurrent_kernel"] = flat(sv["hin"]).T @ flat(dhp)
    grads[f"{p}/hn_bias"] = flat(dhp)[:, 2 * hdim:].sum(0)  # b_hn sits inside r * (.)
    grads[f"{p}/input_kernel"] = flat(cache["gru_in"]).T @ flat(dxp)
    grads[f"{p}/input_bias"] = flat(dxp).sum(0)
    dh = dxp @ wi.T
    for ent in reversed(cache["layers"]):
        layer, lp = ent["layer"], ent["prefix"]
        dz_ = dh * net.activation_grad(ent["z"], ent["h"], layer.activation)
        grads[f"{lp}/kernel"] = flat(ent["x"]).T @ flat(dz_)
        grads[f"{lp}/bias"] = flat(dz_).sum(0)
        dh = dz_ @ params[f"{lp}/kernel"].astype(dtype).T
    return grads


def loss_and_grads(spec, ppo, params, traj, carry, dtype=np.float32):
    """One env-minibatch: traj leaves [B, T, ...] (obs, done, action, log_prob, value,
    advantages, returns); recurrent_ppo.py:101-184 and :227-253."""
    dt = np.dtype(dtype).type
    done = traj["done"]
    out, value, cache = forward_seq(spec, params, traj["obs"], done, carry, dtype)
    b, t = value.shape
    m = b * t
    flat = lambda a: a.reshape(m, *a.shape[2:])
    out_f, value_f = flat(out), flat(value)
    act = flat(traj["action"])
    lp, ent, hc = head_logprob_entropy(spec, out_f, act, params, dt)
    lp_old = flat(traj["log_prob"]).astype(dtype)
    adv = flat(traj["advantages"]).astype(dtype)
    ret = flat(traj["returns"]).astype(dtype)
    v_old = flat(traj["value"]).astype(dtype)
    eps = dt(ppo.clip_coefficient)
    entropy = ent.mean()
    ratio = np.exp(lp - lp_old)
    approx_kl = (lp_old - lp).mean()
    clip_frac = (np.abs(ratio - dt(1)) > eps).astype(dtype).mean()
    dclip_r, clipped = _clip_grad(ratio, dt(1) - eps, dt(1) + eps)
    s1, s2 = ratio * adv, clipped * adv
    mn = np.minimum(s1, s2)
    actor_loss = -mn.mean()
    c1 = dt(0.5) * ((value_f - ret) ** 2)
    if ppo.clip_value_loss:
        dclip_v, cl = _clip_grad(value_f - v_old, -eps, eps)
        vc = v_old + cl
        c2 = dt(0.5) * ((vc - ret) ** 2)
        crit = np.maximum(c1, c2)
        dcrit = _tie(c1, crit, c2) * (value_f - ret) + _tie(c2, crit, c1) * (vc - ret) * dclip_v
    else:
        crit, dcrit = c1, value_f - ret
    critic_loss = crit.mean()
    loss = actor_loss - dt(ppo.entropy_coefficient) * entropy + dt(ppo.value_coefficient) * critic_loss
    resid = ret - value_f
    ev = dt(1) - resid.var() / (ret.var() + dt(1e-8))
    stats = np.array([actor_loss, entropy, approx_kl, clip_frac, adv.mean(), critic_loss, ev,
                      value_f.mean()], np.float64)
    inv_m = dt(1.0 / m)
    t1, t2 = _tie(s1, mn, s2), _tie(s2, mn, s1)
    g_lp = -((t1 * adv + t2 * adv * dclip_r) * ratio) * inv_m
    g_ent = -dt(ppo.entropy_coefficient) * inv_m
    d_value = dt(ppo.value_coefficient) * inv_m * dcrit
    p, logp = hc["p"], hc["logp"]
    onehot = np.zeros_like(p)
    onehot[np.arange(m), act.astype(np.int64)] = 1
    d_out = g_lp[:, None] * (onehot - p) + g_ent * (-p * (logp + ent[:, None]))
    grads = backward_seq(spec, params, cache, d_out.reshape(b, t, -1).astype(dtype),
                         d_value.reshape(b, t).astype(dtype), done, dtype)
    return float(loss), stats, grads


def update(spec, ppo, opt, params, opt_state, rollout, env_perms, dtype=np.float32,
           max_minibatches=None):
    """The full RecurrentPPO learner step of one device. rollout: [T, N] leaves plus
    first_done [T, N], carry [N, H] (entering step 0), last_carry [N, H] (entering T-1),
    bootstrap_obs [N, D]. env_perms: [E, N]."""
    t, n = rollout["reward"].shape
    # tail bootstrap: (first[-1], second[-1]) from the carry entering step T-1
    seq_obs = np.stack([rollout["obs"][-1], rollout["bootstrap_obs"]], axis=1)
    second_done = rollout["terminated"][-1] | rollout["truncated"][-1]
    seq_done = np.stack([rollout["first_done"][-1], second_done], axis=1)
    _, v2, _ = forward_seq(spec, params, seq_obs, seq_done, rollout["last_carry"], dtype)
    boot = v2[:, -1]
    adv, ret = gae_mod.gae(rollout["reward"], rollout["terminated"], rollout["truncated"],
                           rollout["value"], boot, ppo.gamma, ppo.gae_lambda, dtype=dtype)
    if ppo.normalize_advantage:
        adv = (adv - adv.mean()) / (adv.std() + np.dtype(dtype).type(1e-8))
    bt = lambda a: np.moveaxis(a, 0, 1)  # [T, N, ...] -> [N, T, ...]
    seqs = {"obs": bt(rollout["obs"]), "done": bt(rollout["first_done"]),
            "action": bt(rollout["action"]), "log_prob": bt(rollout["log_prob"]),
            "value": bt(rollout["value"]), "advantages": bt(adv), "returns": bt(ret)}
    mbs = ppo.num_minibatches
    stats = np.zeros((ppo.update_epochs, mbs, 8))
    done_steps = 0
    for e in range(ppo.update_epochs):
        idx = np.asarray(env_perms[e]).reshape(mbs, -1)
        for k in range(mbs):
            if max_minibatches is not None and done_steps >= max_minibatches:
                return params, opt_state, stats, {"advantages": adv, "returns": ret, "bootstrap": boot}
            traj = {key: val[idx[k]] for key, val in seqs.items()}
            _, st, grads = loss_and_grads(spec, ppo, params, traj, rollout["carry"][idx[k]], dtype)
            params, opt_state = optim.clip_adam(params, grads, opt_state, opt, dtype)
            stats[e, k] = st
            done_steps += 1
    return params, opt_state, stats, {"advantages": adv, "returns": ret, "bootstrap": boot}
