"""Regenerates tests/golden/gae_kat.npz, the GAE known-answer vectors.

The reference pins GAE with a NumPy-only known-answer test
(boonta tests/test_algorithms.py:103-152): inputs drawn from np.random.default_rng(0) for
a (6, 3) rollout, gamma 0.9, lambda 0.8, terminations and truncations at p = 0.2 (never
both), once with rho = c = 1 ("gae") and once with rho, c ~ U(0.5, 1.5) ("vtrace"); the
expected advantages come from a float64 reverse loop over the recursion, and the JAX
result must match within rtol 1e-5 / atol 1e-6. This script draws the same inputs in the
same order and evaluates the same recursion in float64, so the fixture carries the
reference test's own inputs and expected outputs.

Run: python tests/golden/make_golden.py   (writes gae_kat.npz beside this file)
"""
from pathlib import Path

import numpy as np

GAMMA, LAMBDA = 0.9, 0.8


def expected_advantages(reward, values, bootstrap, terminated, truncated, rho, c):
    advantages = np.zeros_like(values)
    advantage, next_value = np.zeros_like(bootstrap), bootstrap
    for t in reversed(range(len(values))):
        alive = (1.0 - terminated[t]) * (1.0 - truncated[t])
        delta = rho[t] * (reward[t] + GAMMA * (1.0 - terminated[t]) * next_value - values[t])
        delta = delta * (1.0 - truncated[t])
        advantage = delta + GAMMA * LAMBDA * c[t] * alive * advantage
        advantages[t] = advantage
        next_value = values[t]
    return advantages


def case(weighted: bool) -> dict:
    generator = np.random.default_rng(0)
    shape = (6, 3)
    reward, values = generator.normal(size=shape), generator.normal(size=shape)
    bootstrap = generator.normal(size=shape[1:])
    terminated = generator.random(shape) < 0.2
    truncated = (generator.random(shape) < 0.2) & ~terminated
    rho, c = (
        generator.uniform(0.5, 1.5, shape) if weighted else np.ones(shape) for _ in range(2)
    )
    adv = expected_advantages(reward, values, bootstrap, terminated, truncated, rho, c)
    return {
        "reward": reward, "values": values, "bootstrap": bootstrap,
        "terminated": terminated.astype(np.uint8), "truncated": truncated.astype(np.uint8),
        "rho": rho, "c": c, "advantages": adv, "returns": adv + values,
    }


def main():
    out = {}
    for name, weighted in (("gae", False), ("vtrace", True)):
        for key, value in case(weighted).items():
            out[f"{name}/{key}"] = value
    out["gamma"] = np.float64(GAMMA)
    out["gae_lambda"] = np.float64(LAMBDA)
    path = Path(__file__).with_name("gae_kat.npz")
    np.savez(path, **out)
    print(f"wrote {path}")


if __name__ == "__main__":
    main()
