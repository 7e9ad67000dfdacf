"""Network and algorithm specifications for the PPO learner step.

These dataclasses describe, in plain Python, everything the native learner needs to
know about one PPO problem: the hyperparameters (`PPOConfig`, the same field names as
boonta/algorithms/ppo.py:17-27), the optimizer chain
`optax.chain(clip_by_global_norm(max_grad_norm), adam(lr, b1, b2, eps))` used by every
PPO recipe (e.g. hangar/recipes/ppo_cartpole.py:44-47), and the actor-critic network
built by the recipes (hangar/recipes/ppo_*.py) as a list of layers.

The flat parameter layout defined here (`param_layout`) is the one the CUDA learner
uses for params, gradients and both Adam moments. The C++ side computes the same
layout (boonta_b200/csrc/learner.cu, `build_layout`); a CPU test checks that the two
agree through `bt_learner_param_info`.
"""
from __future__ import annotations

import math
from dataclasses import dataclass, field

import numpy as np

# --- layer kinds -------------------------------------------------------------------

ACTIVATIONS = ("none", "tanh", "relu", "silu")


@dataclass(frozen=True)
class Dense:
    """flax.linen.Dense(features) followed by an optional LayerNorm and an activation."""

    features: int
    activation: str = "none"
    layernorm: bool = False


@dataclass(frozen=True)
class Conv3x3:
    """flax.linen.Conv(features, (3, 3), padding="SAME") on an NHWC image, then an
    activation and a flatten in (h, w, c) order (boonta.networks.layers.Flatten)."""

    features: int
    height: int
    width: int
    in_channels: int
    activation: str = "relu"


@dataclass(frozen=True)
class GRU:
    """flax.linen.GRUCell(features) scanned over time by boonta.networks.RNN
    (boonta/networks/blocks/rnn.py:30-54), reset to zeros where `first.done`."""

    features: int


@dataclass(frozen=True)
class NetworkSpec:
    """Actor-critic network: a torso (shared, or the actor's own tower when `critic`
    is given) and heads (boonta/networks/actor_critic.py:7-14)."""

    obs_dim: int
    torso: tuple
    critic: tuple | None = None  # None: the torso is shared by both heads
    head: str = "categorical"  # "categorical" | "gaussian"
    action_dim: int = 2

    @property
    def shared(self) -> bool:
        return self.critic is None

    @property
    def recurrent(self) -> bool:
        return any(isinstance(layer, GRU) for layer in self.torso)

    def towers(self) -> list[tuple]:
        return [self.torso] if self.shared else [self.torso, self.critic]


@dataclass(frozen=True)
class PPOConfig:
    """boonta/algorithms/ppo.py:17-27 (field names and defaults kept)."""

    num_minibatches: int
    update_epochs: int
    clip_coefficient: float
    clip_value_loss: bool
    entropy_coefficient: float
    value_coefficient: float
    gamma: float
    gae_lambda: float
    normalize_advantage: bool = False


@dataclass(frozen=True)
class OptimizerConfig:
    """optax.chain(optax.clip_by_global_norm(max_grad_norm), optax.adam(lr, b1, b2, eps,
    eps_root)) as built by the PPO recipes (hangar/recipes/ppo_cartpole.py:44-47)."""

    lr: float
    max_grad_norm: float = 0.5
    b1: float = 0.9
    b2: float = 0.999
    eps: float = 1e-8
    eps_root: float = 0.0


# --- flat parameter layout -----------------------------------------------------------

ALIGN = 64  # floats: every parameter group starts on a 256-byte boundary


def _align(n: int) -> int:
    return (n + ALIGN - 1) // ALIGN * ALIGN


@dataclass
class ParamEntry:
    name: str
    shape: tuple
    offset: int  # in floats

    @property
    def size(self) -> int:
        return int(np.prod(self.shape)) if self.shape else 1


@dataclass
class ParamLayout:
    entries: list = field(default_factory=list)
    total: int = 0

    def __getitem__(self, name: str) -> ParamEntry:
        for entry in self.entries:
            if entry.name == name:
                return entry
        raise KeyError(name)

    def names(self) -> list[str]:
        return [entry.name for entry in self.entries]

    def unflatten(self, flat: np.ndarray) -> dict:
        return {
            e.name: flat[e.offset : e.offset + e.size].reshape(e.shape).copy()
            for e in self.entries
        }

    def flatten(self, params: dict, dtype=np.float32) -> np.ndarray:
        flat = np.zeros(self.total, dtype)
        for e in self.entries:
            flat[e.offset : e.offset + e.size] = np.asarray(params[e.name], dtype).ravel()
        return flat


def layer_output_dim(layer, in_dim: int) -> int:
    if isinstance(layer, Conv3x3):
        return layer.height * layer.width * layer.features
    return layer.features


def tower_dims(spec: NetworkSpec, tower: tuple) -> list[int]:
    """Input width of every layer of a tower, followed by the tower's output width."""
    dims = [spec.obs_dim]
    for layer in tower:
        dims.append(layer_output_dim(layer, dims[-1]))
    return dims


def param_layout(spec: NetworkSpec) -> ParamLayout:
    """Groups are placed in this order, each group aligned to ALIGN floats:

    for every tower (torso, then critic when separate), for every layer:
      Dense:   kernel [K, N] immediately followed by bias [N]
               (+ a LayerNorm group: scale [N] immediately followed by bias [N])
      Conv3x3: kernel [3, 3, Cin, Cout] immediately followed by bias [Cout]
      GRU:     input kernel [K, 3H] (+ bias [3H]); recurrent kernel [H, 3H]; bias of hn [H]
    then the actor head kernel [F, A] + bias [A], the gaussian scale [A] (gaussian only),
    and the critic head kernel [F, 1] + bias [1].

    Keeping bias right after its kernel makes each Dense a single [K+1, N] matrix, so
    one GEMM with a constant-one input column produces z = x W + b and dW, db together.
    """
    layout = ParamLayout()
    off = 0

    def group(*parts):
        nonlocal off
        for name, shape in parts:
            layout.entries.append(ParamEntry(name, tuple(shape), off))
            off += int(np.prod(shape))
        off = _align(off)

    tower_names = ["torso"] if spec.shared else ["actor", "critic"]
    for tname, tower in zip(tower_names, spec.towers()):
        dims = tower_dims(spec, tower)
        for i, layer in enumerate(tower):
            k = dims[i]
            p = f"{tname}/{i}"
            if isinstance(layer, Dense):
                group((f"{p}/kernel", (k, layer.features)), (f"{p}/bias", (layer.features,)))
                if layer.layernorm:
                    group((f"{p}/ln_scale", (layer.features,)), (f"{p}/ln_bias", (layer.features,)))
            elif isinstance(layer, Conv3x3):
                group(
                    (f"{p}/kernel", (3, 3, layer.in_channels, layer.features)),
                    (f"{p}/bias", (layer.features,)),
                )
            elif isinstance(layer, GRU):
                h = layer.features
                group((f"{p}/input_kernel", (k, 3 * h)), (f"{p}/input_bias", (3 * h,)))
                group((f"{p}/recurrent_kernel", (h, 3 * h)))
                group((f"{p}/hn_bias", (h,)))
            else:
                raise TypeError(layer)
    feat_pi = tower_dims(spec, spec.torso)[-1]
    feat_v = tower_dims(spec, spec.critic)[-1] if not spec.shared else feat_pi
    a = spec.action_dim
    group(("actor_head/kernel", (feat_pi, a)), ("actor_head/bias", (a,)))
    if spec.head == "gaussian":
        group(("actor_head/scale", (a,)))
    group(("critic_head/kernel", (feat_v, 1)), ("critic_head/bias", (1,)))
    layout.total = off
    return layout


# --- initialisers (host side; flax conventions) --------------------------------------


def orthogonal(rng: np.random.Generator, shape, gain: float = 1.0) -> np.ndarray:
    """flax.linen.initializers.orthogonal on a 2-D [fan_in, fan_out] matrix
    (QR of a Gaussian matrix, sign-corrected)."""
    rows, cols = int(np.prod(shape[:-1])), shape[-1]
    n, m = max(rows, cols), min(rows, cols)
    a = rng.standard_normal((n, m))
    q, r = np.linalg.qr(a)
    q = q * np.sign(np.diag(r))
    if rows < cols:
        q = q.T
    return (gain * q[:rows, :cols]).reshape(shape).astype(np.float32)


def lecun_normal(rng: np.random.Generator, shape, fan_in: int) -> np.ndarray:
    """flax default kernel init: truncated normal (within 2 std) with variance 1/fan_in."""
    std = math.sqrt(1.0 / fan_in) / 0.87962566103423978
    out = rng.standard_normal(int(np.prod(shape)))
    bad = np.abs(out) > 2.0
    while bad.any():
        out[bad] = rng.standard_normal(int(bad.sum()))
        bad = np.abs(out) > 2.0
    return (out * std).reshape(shape).astype(np.float32)


def init_params(spec: NetworkSpec, seed: int = 0, init: str = "lecun") -> dict:
    """Random-init weights of the spec's architecture. `init="orthogonal"` uses the
    CleanRL-style gains (sqrt(2) hidden, 0.01 policy head, 1.0 value head)."""
    rng = np.random.default_rng(seed)
    layout = param_layout(spec)
    params = {}
    for e in layout.entries:
        name = e.name
        if name.endswith("ln_scale"):
            params[name] = np.ones(e.shape, np.float32)
        elif name.endswith("/scale"):  # gaussian state-independent scale: std 1 at init
            params[name] = np.full(e.shape, np.log(np.expm1(1.0 - 1e-3)), np.float32)
        elif "bias" in name:
            params[name] = np.zeros(e.shape, np.float32)
        elif name.endswith("recurrent_kernel"):
            h = e.shape[0]
            params[name] = np.concatenate(
                [orthogonal(rng, (h, h)) for _ in range(3)], axis=1
            )
        else:
            fan_in = int(np.prod(e.shape[:-1]))
            if init == "orthogonal":
                gain = 0.01 if name.startswith("actor_head") else (
                    1.0 if name.startswith("critic_head") else math.sqrt(2.0))
                params[name] = orthogonal(rng, e.shape, gain)
            else:
                params[name] = lecun_normal(rng, e.shape, fan_in)
    return params
