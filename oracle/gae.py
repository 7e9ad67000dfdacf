"""Generalized advantage estimation, restated from
boonta/algorithms/advantage_estimators.py:8-56 (test infrastructure only).

The reference runs a reverse `jax.lax.scan` with carry (advantage, next_value) initialised
to (0, bootstrap); each step computes

    delta = rho * (reward + gamma * (1 - terminated) * next_value - value)   # :30
    delta *= 1 - truncated                                                    # :31
    advantage = delta + gamma * gae_lambda * c * (1 - terminated) * (1 - truncated) * advantage
    next_value <- value                                                       # :41

and returns (advantages, advantages + values) (:56). `gamma` and `gae_lambda` are Python
floats in the reference, so `gamma * gae_lambda` is formed in double precision and then
rounded once to float32; every array operation is float32 (dtype = result_type(values,
bootstrap, rewards, float32), :18). The float32 path below keeps that operation order, so
it is bit-identical to a non-fused float32 evaluation of the reference expression.
"""
from __future__ import annotations

import numpy as np


def gae(reward, terminated, truncated, values, bootstrap, gamma, gae_lambda,
        rho=None, c=None, dtype=np.float32):
    reward = np.asarray(reward, dtype)
    values = np.asarray(values, dtype)
    bootstrap = np.asarray(bootstrap, dtype)
    term = 1.0 - np.asarray(terminated, dtype)
    trunc = 1.0 - np.asarray(truncated, dtype)
    term = term.astype(dtype)
    trunc = trunc.astype(dtype)
    rho = np.ones_like(values) if rho is None else np.asarray(rho, dtype)
    c = np.ones_like(values) if c is None else np.asarray(c, dtype)
    g = dtype(gamma)
    gl = dtype(float(gamma) * float(gae_lambda))

    advantages = np.zeros_like(values)
    advantage = np.zeros_like(bootstrap)
    next_value = bootstrap
    for t in reversed(range(values.shape[0])):
        delta = rho[t] * (reward[t] + g * term[t] * next_value - values[t])
        delta = delta * trunc[t]
        advantage = delta + gl * c[t] * term[t] * trunc[t] * advantage
        advantages[t] = advantage
        next_value = values[t]
    return advantages, advantages + values
