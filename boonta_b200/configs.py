"""The five synthetic learner-step workloads (C1-C5) and their seeded input generators.

Each workload stands in for a boonta recipe's rollout (CartPole, Brax, MinAtar, a GRU
agent, Craftax-symbolic) with the shapes and value distributions of that recipe; no
environment or dataset is used. Inputs come from numpy's PCG64 with seeds 0..4, so the
oracle and the CUDA learner see identical bytes.

A `Rollout` holds one learner input in boonta's `Transition` layout, leaves `[T, N, ...]`
(boonta/utils/transition.py:9-26): `first.obs`, `second.{action, reward, terminated,
truncated}`, `aux.{log_prob, value}`, plus `second.obs[-1]` (the bootstrap observation,
boonta/algorithms/ppo.py:208-212). Recurrent workloads add `first.done` and the carry
entering step 0 (`transitions.start`, boonta/algorithms/recurrent_ppo.py:211).
"""
from __future__ import annotations

from dataclasses import dataclass

import numpy as np

from .spec import GRU, Conv3x3, Dense, NetworkSpec, OptimizerConfig, PPOConfig


@dataclass(frozen=True)
class Workload:
    name: str
    description: str
    num_steps: int  # T
    num_envs: int  # N per GPU
    ppo: PPOConfig
    optimizer: OptimizerConfig
    network: NetworkSpec
    precision: str = "fp32"  # GEMM operand precision: fp32 | bf16 | bf16x3
    init: str = "lecun"
    seed: int = 0
    reward: str = "normal"
    done_p: float = 0.01
    obs_kind: str = "normal"
    obs_sparsity: float = 0.0
    reward_scale: float = 1.0
    reward_p: float = 0.05
    hidden_std: float = 0.1

    @property
    def batch_size(self) -> int:
        return self.num_steps * self.num_envs

    @property
    def minibatch_size(self) -> int:
        if self.network.recurrent:
            return self.num_envs // self.ppo.num_minibatches
        return self.batch_size // self.ppo.num_minibatches

    def scaled(self, num_steps: int | None = None, num_envs: int | None = None,
               num_minibatches: int | None = None, update_epochs: int | None = None) -> "Workload":
        """The same network and losses on a smaller rollout (for oracle-sized tests)."""
        import dataclasses

        ppo = self.ppo
        if num_minibatches is not None or update_epochs is not None:
            ppo = dataclasses.replace(
                ppo,
                num_minibatches=num_minibatches or ppo.num_minibatches,
                update_epochs=update_epochs or ppo.update_epochs,
            )
        return dataclasses.replace(
            self, num_steps=num_steps or self.num_steps, num_envs=num_envs or self.num_envs, ppo=ppo
        )


def _ppo(gamma, lam, clip, epochs, minibatches, ent=0.01, vf=0.5):
    # Defaults from hangar/config/algorithm/ppo.yaml:4-13 (clip_value_loss True,
    # normalize_advantage False); each workload overrides gamma/lambda/clip/E/M.
    return PPOConfig(
        num_minibatches=minibatches,
        update_epochs=epochs,
        clip_coefficient=clip,
        clip_value_loss=True,
        entropy_coefficient=ent,
        value_coefficient=vf,
        gamma=gamma,
        gae_lambda=lam,
        normalize_advantage=False,
    )


def c1() -> Workload:
    """CartPole-shaped (hangar/recipes/ppo_cartpole.py:24-47): 4->64->64 tanh, shared."""
    return Workload(
        name="c1_cartpole",
        description="T=128 x N=16, MLP 4-64-64 tanh, categorical(2), 4x4 minibatches, fp32",
        num_steps=128, num_envs=16,
        ppo=_ppo(0.99, 0.95, 0.2, 4, 4),
        optimizer=OptimizerConfig(lr=2.5e-4, max_grad_norm=0.5, eps=1e-5),
        network=NetworkSpec(
            obs_dim=4,
            torso=(Dense(64, "tanh"), Dense(64, "tanh")),
            head="categorical", action_dim=2,
        ),
        init="orthogonal", seed=0, reward="ones", done_p=0.02,
    )


def c2(precision: str = "bf16x3") -> Workload:
    """Brax-shaped (hangar/recipes/ppo_mujoco.py:16-31): separate actor and critic towers
    87->256->256->256 SiLU, gaussian head with a learned state-independent scale. "fp32
    params with TF32/bf16 GEMMs allowed within the stated tolerance": split-bf16 tensor-core
    GEMMs by default (fp32-accurate to ~1e-5 per product)."""
    tower = (Dense(256, "silu"), Dense(256, "silu"), Dense(256, "silu"))
    return Workload(
        name="c2_brax",
        description="T=64 x N=8192, actor+critic 87-256-256-256 SiLU, gaussian(8), 4x32 minibatches",
        num_steps=64, num_envs=8192,
        ppo=_ppo(0.97, 0.95, 0.3, 4, 32),
        optimizer=OptimizerConfig(lr=3e-4, max_grad_norm=0.5),
        network=NetworkSpec(obs_dim=87, torso=tower, critic=tower, head="gaussian", action_dim=8),
        precision=precision, seed=1, reward="normal", done_p=0.001,
    )


def c3(precision: str = "fp32") -> Workload:
    """MinAtar-shaped (hangar/recipes/ppo_minatar.py:110-120) with SAME padding: conv 16@3x3
    ReLU -> flatten 1600 -> 128 ReLU, categorical(6), in its stated fp32 arithmetic (every
    layer is narrower than 256 outputs: CUDA-core kernels). The split-bf16 tensor-core option
    for the 1600 -> 128 layer stays available (precision="bf16x3"): on the full 65,536-row
    minibatch its ~1e-5 per-product error flips the ReLU derivative of pre-activations within
    that distance of zero often enough to put the layer's gradients at ~2e-4 of the exact ones,
    above the 1e-4 bound, so it is not the default."""
    return Workload(
        name="c3_minatar",
        description="T=128 x N=4096, conv16 3x3 SAME -> 1600 -> 128 ReLU, categorical(6), 4x8",
        num_steps=128, num_envs=4096,
        ppo=_ppo(0.99, 0.95, 0.2, 4, 8),
        optimizer=OptimizerConfig(lr=5e-4, max_grad_norm=0.5),
        network=NetworkSpec(
            obs_dim=400,
            torso=(Conv3x3(16, 10, 10, 4, "relu"), Dense(128, "relu")),
            head="categorical", action_dim=6,
        ),
        precision=precision, seed=2, reward="bernoulli", reward_p=0.05, done_p=0.01,
        obs_kind="bernoulli",
        obs_sparsity=0.9,
    )


def c4() -> Workload:
    """Recurrent (hangar/recipes/recurrent_ppo_minatar.py, linear encoder): 64->256 ReLU ->
    GRU 256 -> categorical(8); env-minibatches with full-sequence BPTT."""
    return Workload(
        name="c4_gru",
        description="T=128 x N=2048, 64-256 ReLU -> GRU256, categorical(8), 2x8 env-minibatches",
        num_steps=128, num_envs=2048,
        ppo=_ppo(0.99, 0.95, 0.2, 2, 8),
        optimizer=OptimizerConfig(lr=3e-4, max_grad_norm=0.5),
        network=NetworkSpec(
            obs_dim=64, torso=(Dense(256, "relu"), GRU(256)), head="categorical", action_dim=8,
        ),
        seed=3, reward="normal", done_p=0.02,
    )


def c5(precision: str = "bf16") -> Workload:
    """Craftax-symbolic-shaped scaling workload: 8268->512->512->512 LayerNorm+ReLU,
    categorical(43), bf16 GEMM operands with fp32 accumulation and fp32 master params."""
    tower = tuple(Dense(512, "relu", layernorm=True) for _ in range(3))
    return Workload(
        name="c5_craftax",
        description="T=64 x N=4096, MLP 8268-512x3 LN+ReLU, categorical(43), 4x16, bf16 GEMMs",
        num_steps=64, num_envs=4096,
        ppo=_ppo(0.999, 0.8, 0.2, 4, 16),
        optimizer=OptimizerConfig(lr=2e-4, max_grad_norm=0.5),
        network=NetworkSpec(obs_dim=8268, torso=tower, head="categorical", action_dim=43),
        precision=precision, seed=4, reward="normal", reward_scale=0.1, done_p=0.005,
        obs_kind="sparse_uniform", obs_sparsity=0.9,
    )


WORKLOADS = {"c1": c1, "c2": c2, "c3": c3, "c4": c4, "c5": c5}


def make(name: str, **kwargs) -> Workload:
    return WORKLOADS[name](**kwargs)


# --- synthetic rollouts ----------------------------------------------------------------


def _obs(rng, w: Workload, shape):
    if w.obs_kind == "bernoulli":
        return (rng.random(shape, dtype=np.float32) < (1.0 - w.obs_sparsity)).astype(np.float32)
    if w.obs_kind == "sparse_uniform":
        x = rng.random(shape, dtype=np.float32)
        keep = rng.random(shape, dtype=np.float32) >= w.obs_sparsity
        return np.where(keep, x, np.float32(0.0)).astype(np.float32)
    return rng.standard_normal(shape, dtype=np.float32)


def rollout(w: Workload, seed: int | None = None, include_obs: bool = True) -> dict:
    """One seeded learner input (numpy arrays, host memory). With `include_obs=False` the
    `[T, N, D]` observations are left out (the caller makes them elsewhere, e.g. on the
    device for a rollout too large for host-side checking); the other leaves then come from
    a different point of the random stream."""
    rng = np.random.default_rng(w.seed if seed is None else seed)
    t, n, d = w.num_steps, w.num_envs, w.network.obs_dim
    a = w.network.action_dim
    out = {}
    if include_obs:
        out["obs"] = _obs(rng, w, (t, n, d))
    out["bootstrap_obs"] = _obs(rng, w, (n, d))
    if w.network.head == "gaussian":
        out["action"] = rng.standard_normal((t, n, a), dtype=np.float32)
        base = (-0.5 * out["action"] ** 2 - 0.5 * np.log(2 * np.pi)).sum(-1)
        out["log_prob"] = (base + 0.05 * rng.standard_normal((t, n))).astype(np.float32)
    else:
        out["action"] = rng.integers(0, a, (t, n), dtype=np.int32)
        out["log_prob"] = (np.log(1.0 / a) + 0.05 * rng.standard_normal((t, n))).astype(np.float32)
    if w.reward == "ones":
        out["reward"] = np.ones((t, n), np.float32)
    elif w.reward == "bernoulli":
        out["reward"] = (rng.random((t, n)) < w.reward_p).astype(np.float32)
    else:
        out["reward"] = (w.reward_scale * rng.standard_normal((t, n))).astype(np.float32)
    out["terminated"] = (rng.random((t, n)) < w.done_p).astype(np.uint8)
    out["truncated"] = np.zeros((t, n), np.uint8)
    out["value"] = rng.standard_normal((t, n), dtype=np.float32)
    if w.network.recurrent:
        h = [layer for layer in w.network.torso if isinstance(layer, GRU)][0].features
        first_done = np.zeros((t, n), np.uint8)
        first_done[0] = (rng.random(n) < w.done_p).astype(np.uint8)
        first_done[1:] = out["terminated"][:-1] | out["truncated"][:-1]
        out["first_done"] = first_done
        out["carry"] = (w.hidden_std * rng.standard_normal((n, h))).astype(np.float32)
        # boonta's RecurrentPPO replays the carry entering the last step for the tail
        # bootstrap (transitions.tail(), boonta/utils/transition.py:20-26); the synthetic
        # rollout carries it as an explicit input.
        out["last_carry"] = (w.hidden_std * rng.standard_normal((n, h))).astype(np.float32)
        out["bootstrap_done"] = out["terminated"][-1] | out["truncated"][-1]
    return out


def permutations(w: Workload, seed: int | None = None, num_ranks: int = 1) -> np.ndarray:
    """Minibatch permutations, one per epoch: `[E, B_global]` int32 over the global batch
    (flat index t*N_global + n) or, for recurrent workloads, `[E, N_global]` over envs.
    They replace `jax.random.permutation(key, batch_size)` (boonta/algorithms/ppo.py:200)
    as an explicit input."""
    rng = np.random.default_rng(1000 + (w.seed if seed is None else seed))
    size = w.num_envs * num_ranks if w.network.recurrent else w.batch_size * num_ranks
    return np.stack([rng.permutation(size).astype(np.int32) for _ in range(w.ppo.update_epochs)])
