"""clip_by_global_norm + Adam + apply_updates (test infrastructure only).

Restates optax 0.2.8 (third-party, not vendored, not installed) as called by the PPO
recipes: `optax.chain(optax.clip_by_global_norm(max_norm), optax.adam(lr, b1, b2, eps,
eps_root))` and `optax.apply_updates` (boonta/algorithms/ppo.py:182-191,
hangar/recipes/ppo_cartpole.py:44-47). The update rule is Kingma & Ba (2015) with
optax's documented conventions:

    g_norm  = sqrt(sum over all leaves of sum(g^2))
    g       = g                          if g_norm < max_norm
              (g / g_norm) * max_norm    otherwise
    mu      = (1 - b1) * g   + b1 * mu
    nu      = (1 - b2) * g^2 + b2 * nu
    count   = count + 1                   (int32)
    mu_hat  = mu / (1 - b1**count)
    nu_hat  = nu / (1 - b2**count)
    u       = -lr * mu_hat / (sqrt(nu_hat + eps_root) + eps)
    p       = p + u

Parity is unpinned against optax itself (no optax in the image); it follows this rule.
"""
from __future__ import annotations

import numpy as np


def clip_adam(params: dict, grads: dict, state: dict, opt, dtype=np.float32):
    """Returns (new_params, new_state). state = {"count": int, "mu": dict, "nu": dict}."""
    dt = np.dtype(dtype).type
    sq = sum(float(np.sum(np.asarray(g, np.float64) ** 2)) for g in grads.values())
    g_norm = dt(np.sqrt(sq))
    max_norm = dt(opt.max_grad_norm)
    count = state["count"] + 1
    b1, b2 = dt(opt.b1), dt(opt.b2)
    bc1 = dt(1) - dt(opt.b1) ** dt(count)
    bc2 = dt(1) - dt(opt.b2) ** dt(count)
    new_params, mu, nu = {}, {}, {}
    for name, g in grads.items():
        g = np.asarray(g, dtype)
        if not g_norm < max_norm:
            g = (g / g_norm) * max_norm
        m = (dt(1) - b1) * g + b1 * state["mu"][name]
        v = (dt(1) - b2) * (g * g) + b2 * state["nu"][name]
        m_hat = m / bc1
        v_hat = v / bc2
        u = dt(-opt.lr) * (m_hat / (np.sqrt(v_hat + dt(opt.eps_root)) + dt(opt.eps)))
        new_params[name] = (np.asarray(params[name], dtype) + u).astype(dtype)
        mu[name], nu[name] = m.astype(dtype), v.astype(dtype)
    return new_params, {"count": count, "mu": mu, "nu": nu, "g_norm": float(g_norm)}


def init_state(params: dict, dtype=np.float32) -> dict:
    return {
        "count": 0,
        "mu": {k: np.zeros_like(np.asarray(v, dtype)) for k, v in params.items()},
        "nu": {k: np.zeros_like(np.asarray(v, dtype)) for k, v in params.items()},
    }
