"""boonta's PPO / RecurrentPPO `Algorithm` API over the native learner.

The classes keep the reference's names, constructor arguments and methods
(boonta/algorithms/algorithm.py:8-20; ppo.py:17-233; recurrent_ppo.py:18-281) so that a
caller written against them keeps its shape:

    ppo = PPO(cfg, network, optimizer)          # ppo.py:37-43
    state, carry = ppo.init(key, timestep)      # ppo.py:45-55
    state, carry, action, aux = ppo.step(state, carry, key, timestep, temperature)
    state = ppo.update(state, key, transitions) # ppo.py:76-233

What changes is the representation. `network` is a `boonta_b200.spec.NetworkSpec` (the
MLP / conv / GRU families the learner implements) instead of a flax module, `optimizer`
is an `OptimizerConfig` describing optax.chain(clip_by_global_norm, adam) instead of an
optax object, and arrays are torch CUDA tensors. `PPOState.params` is the flat parameter
buffer (layout `spec.param_layout`), `optimizer_state` an `AdamState(mu, nu, count)`.
Keys are threefry keys (two uint32 words, as jax.random.key_data returns; an integer seed is
taken as jax.random.PRNGKey(seed)): the permutations (ppo.py:200, 230) and the sampling draws
(ppo.py:68, distributions.py:21-23) are drawn from them on the device in jax.random's
conventions (boonta_b200.random; csrc/random.cu). Parameter initialisation (init) stays a
seeded host draw. Anything the learner does not
implement (auxiliary losses, another advantage estimator, other network modules) raises
NotImplementedError. Every update and act step runs in the CUDA library; there is no CPU
path.
"""
from __future__ import annotations

from dataclasses import dataclass, field, replace
from typing import Any, Callable

import torch

from . import random as trandom
from .spec import NetworkSpec, OptimizerConfig, PPOConfig, init_params, param_layout

RecurrentPPOConfig = PPOConfig  # recurrent_ppo.py:18-28 has the same fields and defaults


@dataclass(frozen=True)
class Timestep:
    """boonta/utils/timestep.py:8-37 (leaves are CUDA tensors, leading axes [T, N] or [N])."""

    obs: Any
    action: Any = None
    reward: Any = None
    terminated: Any = None
    truncated: Any = None
    info: Any = None

    @property
    def done(self):
        return self.terminated.bool() | self.truncated.bool()


@dataclass(frozen=True)
class Transition:
    """boonta/utils/transition.py:9-26: `first` and `second` timesteps of every step, the
    acting-time `aux` ({"log_prob", "value"}) and, for recurrent networks, the carry
    entering every step ([T, N, H])."""

    first: Timestep | None = None
    second: Timestep | None = None
    aux: dict | None = None
    carry: Any = None

    @property
    def start(self):
        return self.carry[0]


@dataclass(frozen=True)
class AdamState:
    """optax adam state of the flat parameter buffer (ScaleByAdamState mu, nu, count); count
    is an int32 device scalar after an update (an int is accepted on the way in). The optax
    chain's pytree (EmptyState, ScaleByAdamState, EmptyState) is boonta_b200.checkpoint's
    state_pytree."""

    mu: torch.Tensor
    nu: torch.Tensor
    count: Any = 0


@dataclass(frozen=True)
class PPOState:
    """ppo.py:30-34."""

    step: torch.Tensor
    params: torch.Tensor
    optimizer_state: AdamState


RecurrentPPOState = PPOState  # recurrent_ppo.py:31-35


def generalized_advantage_estimator(transitions: Transition, values, bootstrap, gamma: float,
                                    gae_lambda: float, rho=1.0, c=1.0):
    """advantage_estimators.py:8-56 on CUDA tensors: (advantages, returns), each [T, N]."""
    from .learner import gae

    s = transitions.second
    shape = s.reward.shape
    dev = s.reward.device

    def full(x):
        if x is None or isinstance(x, (int, float)):
            return None if x in (None, 1.0) else torch.full(shape, float(x), device=dev)
        return x.to(dev, torch.float32).contiguous()

    return gae(s.reward.to(torch.float32).contiguous(), _u8(s.terminated), _u8(s.truncated),
               values.to(torch.float32).contiguous(), bootstrap.to(torch.float32).contiguous(),
               gamma, gae_lambda, rho=full(rho), c=full(c))


def _u8(x):
    return (x if x.dtype == torch.uint8 else x.to(torch.uint8)).contiguous()


def _act_noise(key, network, n: int, device) -> torch.Tensor:
    """The draws behind the act step's sample, from the step key on the device: the uniforms
    of jax.random.gumbel (minval = the smallest normal float32) for a categorical head
    (distributions.py:21-23), standard normals for a gaussian one, [n, action_dim]."""
    a = network.action_dim
    if network.head == "categorical":
        return trandom.uniform(key, (n, a), torch.finfo(torch.float32).tiny, 1.0, device)
    return trandom.normal(key, (n, a), device)


def _seed(key) -> int:
    if isinstance(key, torch.Tensor):
        return int(key.reshape(-1)[-1].item()) & 0x7FFFFFFFFFFFFFFF
    return int(key) & 0x7FFFFFFFFFFFFFFF


def _flat(x, n: int):
    """[T, N, ...] -> [T*N, n] contiguous float view."""
    return x.reshape(-1, n).to(torch.float32).contiguous()


@dataclass
class PPO:
    """ppo.py:37-43. `precision` picks the learner's GEMM arithmetic ("fp32", "bf16",
    "bf16x3"); it has no counterpart in the reference, where the flax module's dtype
    decides."""

    cfg: PPOConfig
    network: NetworkSpec
    optimizer: OptimizerConfig
    auxiliary_losses: tuple[Callable, ...] = ()
    advantage_estimator: Callable = generalized_advantage_estimator
    precision: str = "fp32"
    init_scheme: str = "lecun"
    _learners: dict = field(default_factory=dict, init=False, repr=False)
    _loaded: dict = field(default_factory=dict, init=False, repr=False)
    metrics: torch.Tensor | None = field(default=None, init=False, repr=False)

    recurrent = False

    def __post_init__(self):
        if not isinstance(self.network, NetworkSpec):
            raise NotImplementedError(
                f"network {type(self.network).__name__}: the learner implements "
                "boonta_b200.spec.NetworkSpec (Dense / Conv3x3 / GRU towers) only")
        if self.network.recurrent != self.recurrent:
            raise NotImplementedError(
                "recurrent networks train through RecurrentPPO" if self.network.recurrent
                else "RecurrentPPO needs a GRU torso")
        if self.auxiliary_losses:
            raise NotImplementedError("auxiliary losses are not part of the native learner")
        if self.advantage_estimator is not generalized_advantage_estimator:
            raise NotImplementedError("the native learner implements the GAE estimator only")
        if not isinstance(self.optimizer, OptimizerConfig):
            raise NotImplementedError(
                "optimizer: an OptimizerConfig (clip_by_global_norm + adam) is expected")

    # ---- learners (one per rollout shape) -------------------------------------------------
    def _learner(self, num_steps: int, num_envs: int):
        from .learner import Learner

        key = (num_steps, num_envs)
        if key not in self._learners:
            self._learners[key] = Learner(self.network, self.cfg, self.optimizer, num_steps,
                                          num_envs, precision=self.precision)
        return self._learners[key]

    @staticmethod
    def _tag(state: PPOState):
        opt = state.optimizer_state
        count = opt.count if isinstance(opt.count, int) else id(opt.count)
        return (id(state.params), id(opt.mu), id(opt.nu), count)

    def _load(self, lrn, state: PPOState):
        """Brings the handle to `state` unless it already holds it (device copies only)."""
        tag = self._tag(state)
        if self._loaded.get(id(lrn)) != tag:
            opt = state.optimizer_state
            count = opt.count
            if not isinstance(count, torch.Tensor):
                count = torch.tensor(int(count), dtype=torch.int32)
            lrn.load_state(state.params.to(lrn.device, torch.float32), opt.mu.to(lrn.device),
                           opt.nu.to(lrn.device), count.to(lrn.device))
            self._loaded[id(lrn)] = tag

    # ---- Algorithm protocol ---------------------------------------------------------------
    def init(self, key, timestep: Timestep):
        """ppo.py:45-55: parameters from the network's initialisers, zero Adam moments."""
        layout = param_layout(self.network)
        dev = timestep.obs.device if isinstance(timestep.obs, torch.Tensor) else "cuda"
        params = torch.as_tensor(layout.flatten(init_params(self.network, seed=_seed(key),
                                                            init=self.init_scheme)),
                                 dtype=torch.float32, device=dev)
        state = PPOState(step=torch.zeros((), dtype=torch.int64),
                         params=params,
                         optimizer_state=AdamState(torch.zeros_like(params),
                                                   torch.zeros_like(params), 0))
        return state, None

    def step(self, state: PPOState, carry, key, timestep: Timestep, temperature: float = 1.0):
        """ppo.py:57-74: act on timestep.obs [N, ...]; returns (state, carry, action,
        {"log_prob", "value"})."""
        obs = _flat(timestep.obs, self.network.obs_dim)
        n = obs.shape[0]
        lrn = self._act_learner(n)
        self._load(lrn, state)
        noise = _act_noise(key, self.network, n, obs.device)
        action, log_prob, value = lrn.act(obs, noise, temperature)
        return state, carry, action, {"log_prob": log_prob, "value": value}

    def _act_learner(self, n: int):
        for (t, envs), lrn in self._learners.items():
            if envs >= n:
                return lrn
        return self._learner(1, n)

    def _permutations(self, key, batch: int, device) -> torch.Tensor:
        """One permutation of the batch per epoch, drawn on the device from the update key as
        the reference does: keys = split(key, update_epochs), permutation(keys[e], batch)
        (ppo.py:199-203, 230)."""
        keys = trandom.split(key, self.cfg.update_epochs)
        return torch.stack([trandom.permutation(k, batch, device) for k in keys])

    def _batch(self, transitions: Transition) -> dict:
        f, s, aux = transitions.first, transitions.second, transitions.aux
        d = self.network.obs_dim
        batch = {
            "obs": _flat(f.obs, d),
            "bootstrap_obs": _flat(s.obs[-1], d),
            "reward": s.reward.to(torch.float32).contiguous(),
            "terminated": _u8(s.terminated),
            "truncated": _u8(s.truncated),
            "log_prob": aux["log_prob"].to(torch.float32).contiguous(),
            "value": aux["value"].to(torch.float32).contiguous(),
        }
        if self.network.head == "categorical":
            batch["action"] = s.action.to(torch.int32).contiguous()
        else:
            batch["action"] = s.action.to(torch.float32).contiguous()
        return batch

    def update(self, state: PPOState, key, transitions: Transition) -> PPOState:
        """ppo.py:76-233: bootstrap, GAE, update_epochs x num_minibatches minibatch steps.
        The per-minibatch statistics (ppo.py:167-179) are left in `self.metrics`
        ([E, M, 8]) instead of being logged."""
        t, n = transitions.second.reward.shape[:2]
        lrn = self._learner(t, n)
        self._load(lrn, state)
        batch = self._batch(transitions)
        perms = self._permutations(key, self._perm_size(t, n), batch["reward"].device)
        self.metrics = lrn.update(batch, perms)
        # the new state in fresh device buffers (the old state stays valid, as in JAX), copied
        # on the stream with no host synchronisation
        params, mu, nu, count = lrn.store_state()
        new = replace(state, step=state.step, params=params,
                      optimizer_state=AdamState(mu, nu, count))
        self._loaded[id(lrn)] = self._tag(new)
        return new

    def _perm_size(self, t: int, n: int) -> int:
        return t * n


@dataclass
class RecurrentPPO(PPO):
    """recurrent_ppo.py:38-281: env-minibatches of whole sequences, the GRU carry reset on
    `first.done`, the tail bootstrap from the carry entering the last step, and BPTT."""

    recurrent = True

    def init(self, key, timestep: Timestep):
        """recurrent_ppo.py:46-70: also returns the initial carry (zeros [N, H], flax's
        GRUCell.initialize_carry)."""
        state, _ = super().init(key, timestep)
        hidden = self.network.torso[-1].features
        n = timestep.reward.shape[0]
        carry = torch.zeros((n, hidden), dtype=torch.float32, device=state.params.device)
        return state, carry

    def step(self, state, carry, key, timestep, temperature: float = 1.0):
        """recurrent_ppo.py:72-96: one step of the network on timestep.obs [N, ...] from
        `carry` [N, H], zeroed first where the timestep starts an episode (terminated or
        truncated set, boonta/networks/blocks/rnn.py:42-45). Returns (state, new carry,
        action, {"log_prob", "value"})."""
        obs = _flat(timestep.obs, self.network.obs_dim)
        n = obs.shape[0]
        lrn = self._act_learner(n)
        self._load(lrn, state)
        reset = torch.zeros(n, dtype=torch.uint8, device=obs.device)
        for flag in (timestep.terminated, timestep.truncated):
            if flag is not None:
                reset |= torch.as_tensor(flag, device=obs.device).reshape(n).to(torch.uint8)
        noise = _act_noise(key, self.network, n, obs.device)
        action, log_prob, value, new_carry = lrn.act_recurrent(obs, reset, carry, noise,
                                                               temperature)
        return state, new_carry, action, {"log_prob": log_prob, "value": value}

    def _perm_size(self, t: int, n: int) -> int:
        return n  # recurrent_ppo.py:270-276 permutes environments

    def _batch(self, transitions: Transition) -> dict:
        batch = super()._batch(transitions)
        f = transitions.first
        batch["first_done"] = (f.terminated.bool() | f.truncated.bool()).to(torch.uint8).contiguous()
        batch["carry"] = transitions.carry[0].to(torch.float32).contiguous()
        batch["last_carry"] = transitions.carry[-1].to(torch.float32).contiguous()
        return batch
