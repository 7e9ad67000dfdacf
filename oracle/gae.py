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


CHUNKS = 8


def gae_chunked(reward, terminated, truncated, values, bootstrap, gamma, gae_lambda,
                rho=None, c=None):
    """float32 GAE in the CUDA kernel's order (boonta_b200/csrc/gae.cu, gae_chunked_kernel):
    the same per-step terms delta_t, k_t (A_t = delta_t + k_t A_{t+1}), the T steps in 8 chunks
    of ceil(T / 8), each chunk folded from its last step into the map A = M * A_entering + C
    from a zero carry, the maps of the later chunks composed onto the zero advantage past the
    last step, then each chunk rescanned. Every product and sum rounded to float32."""
    f = np.float32
    reward = np.asarray(reward, f)
    values = np.asarray(values, f)
    bootstrap = np.asarray(bootstrap, f)
    term = (1.0 - np.asarray(terminated, f)).astype(f)
    trunc = (1.0 - np.asarray(truncated, f)).astype(f)
    rho = np.ones_like(values) if rho is None else np.asarray(rho, f)
    c = np.ones_like(values) if c is None else np.asarray(c, f)
    g = f(gamma)
    gl = f(float(gamma) * float(gae_lambda))
    T = values.shape[0]
    nxt = np.concatenate([values[1:], bootstrap[None]], axis=0) if T else values
    delta = (rho * (reward + g * term * nxt - values)) * trunc
    k = gl * c * term * trunc
    L = -(-T // CHUNKS) if T else 0
    spans = [(min(T, w * L), min(T, w * L + L)) for w in range(CHUNKS)]
    maps = []
    for t0, t1 in spans:
        M = np.ones_like(bootstrap)
        C = np.zeros_like(bootstrap)
        for t in range(t1 - 1, t0 - 1, -1):
            C = (delta[t] + k[t] * C).astype(f)
            M = (k[t] * M).astype(f)
        maps.append((M, C))
    adv_out = np.zeros_like(values)
    for w, (t0, t1) in enumerate(spans):
        a = np.zeros_like(bootstrap)
        for cc in range(CHUNKS - 1, w, -1):
            M, C = maps[cc]
            a = (M * a + C).astype(f)
        for t in range(t1 - 1, t0 - 1, -1):
            a = (delta[t] + k[t] * a).astype(f)
            adv_out[t] = a
    return adv_out, (adv_out + values).astype(f)
