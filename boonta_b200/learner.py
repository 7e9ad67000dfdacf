"""Host-side handle of the native learner (one per GPU).

`Learner` owns a `bt_learner` from the C-ABI and passes it torch CUDA tensors (torch is
only the device-memory/stream plumbing here). Everything it computes runs in the CUDA
library; there is no CPU path.
"""
from __future__ import annotations

import ctypes as C

import numpy as np
import torch

from . import _lib
from .configs import Workload
from .spec import GRU, Conv3x3, Dense, NetworkSpec, OptimizerConfig, PPOConfig, param_layout

BATCH_FIELDS = ("obs", "bootstrap_obs", "action", "reward", "terminated", "truncated",
                "log_prob", "value", "first_done", "carry", "last_carry")


def _layer_c(layer) -> _lib.Layer:
    c = _lib.Layer()
    if isinstance(layer, Dense):
        c.kind = _lib.BT_LAYER_DENSE
        c.features = layer.features
        c.activation = _lib.ACT[layer.activation]
        c.layernorm = int(layer.layernorm)
    elif isinstance(layer, Conv3x3):
        c.kind = _lib.BT_LAYER_CONV3X3
        c.features = layer.features
        c.activation = _lib.ACT[layer.activation]
        c.height, c.width, c.in_channels = layer.height, layer.width, layer.in_channels
    elif isinstance(layer, GRU):
        c.kind = _lib.BT_LAYER_GRU
        c.features = layer.features
    else:
        raise TypeError(layer)
    return c


def network_c(spec: NetworkSpec) -> _lib.Network:
    n = _lib.Network()
    n.obs_dim = spec.obs_dim
    n.num_torso = len(spec.torso)
    for i, layer in enumerate(spec.torso):
        n.torso[i] = _layer_c(layer)
    n.num_critic = 0 if spec.shared else len(spec.critic)
    if not spec.shared:
        for i, layer in enumerate(spec.critic):
            n.critic[i] = _layer_c(layer)
    n.head = _lib.HEAD[spec.head]
    n.action_dim = spec.action_dim
    return n


def learner_config(network: NetworkSpec, ppo: PPOConfig, opt: OptimizerConfig, num_steps: int,
                   num_envs: int, precision: str = "fp32", world_size: int = 1,
                   rank: int = 0) -> _lib.LearnerConfig:
    cfg = _lib.LearnerConfig()
    cfg.network = network_c(network)
    cfg.ppo = _lib.PPOConfigC(
        ppo.num_minibatches, ppo.update_epochs, ppo.clip_coefficient, int(ppo.clip_value_loss),
        ppo.entropy_coefficient, ppo.value_coefficient, ppo.gamma, ppo.gae_lambda,
        int(ppo.normalize_advantage),
    )
    cfg.optimizer = _lib.OptimizerC(opt.lr, opt.max_grad_norm, opt.b1, opt.b2, opt.eps, opt.eps_root)
    cfg.num_steps, cfg.num_envs = num_steps, num_envs
    cfg.precision = _lib.PRECISION[precision]
    cfg.world_size, cfg.rank = world_size, rank
    return cfg


def _ptr(t: torch.Tensor | None) -> int | None:
    if t is None:
        return None
    if not t.is_cuda:
        raise ValueError("expected a CUDA tensor")
    if not t.is_contiguous():
        raise ValueError("expected a contiguous tensor")
    return t.data_ptr()


def _stream() -> int:
    return torch.cuda.current_stream().cuda_stream


class Learner:
    """One native learner: PPO.update / RecurrentPPO.update on this GPU."""

    def __init__(self, network: NetworkSpec, ppo: PPOConfig, optimizer: OptimizerConfig,
                 num_steps: int, num_envs: int, precision: str = "fp32", world_size: int = 1,
                 rank: int = 0):
        self.network, self.ppo, self.optimizer = network, ppo, optimizer
        self.num_steps, self.num_envs = num_steps, num_envs
        self.world_size, self.rank = world_size, rank
        self.precision = precision
        self._cfg = learner_config(network, ppo, optimizer, num_steps, num_envs, precision,
                                   world_size, rank)
        L = _lib.lib()
        handle = C.c_void_p()
        _lib.check(L.bt_learner_create(C.byref(self._cfg), C.byref(handle)))
        self._h = handle
        self.layout = param_layout(network)
        self.num_params = int(L.bt_learner_num_params(self._h))
        self.device = torch.device("cuda", torch.cuda.current_device())

    @classmethod
    def from_workload(cls, w: Workload, world_size: int = 1, rank: int = 0, **overrides):
        kw = dict(precision=w.precision)
        kw.update(overrides)
        return cls(w.network, w.ppo, w.optimizer, w.num_steps, w.num_envs,
                   world_size=world_size, rank=rank, **kw)

    @property
    def handle(self) -> int:
        """Address of the native bt_learner (the "learner" attribute of the XLA FFI calls)."""
        return int(self._h.value)

    def close(self):
        if getattr(self, "_h", None):
            _lib.lib().bt_learner_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    # ---- layout / state ------------------------------------------------------------------
    def native_layout(self) -> list[tuple[str, int, tuple]]:
        L = _lib.lib()
        out = []
        name = C.create_string_buffer(128)
        off, nd = C.c_int64(), C.c_int32()
        shape = (C.c_int64 * 4)()
        for i in range(L.bt_learner_param_count(self._h)):
            _lib.check(L.bt_learner_param_info(self._h, i, name, 128, C.byref(off), C.byref(nd), shape))
            out.append((name.value.decode(), off.value, tuple(shape[j] for j in range(nd.value))))
        return out

    def set_state(self, params, mu=None, nu=None, count: int = 0):
        """params/mu/nu: dict name -> array, or flat tensors/arrays of num_params floats."""
        def flat(x):
            if x is None:
                return None
            if isinstance(x, dict):
                x = self.layout.flatten(x)
            t = torch.as_tensor(np.asarray(x, np.float32) if not torch.is_tensor(x) else x)
            return t.to(self.device, torch.float32).contiguous()

        p, m, v = flat(params), flat(mu), flat(nu)
        _lib.check(_lib.lib().bt_learner_set_state(self._h, _ptr(p), _ptr(m), _ptr(v), count, _stream()))

    def get_state(self):
        p = torch.empty(self.num_params, dtype=torch.float32, device=self.device)
        m, v = torch.empty_like(p), torch.empty_like(p)
        count = C.c_int32()
        _lib.check(_lib.lib().bt_learner_get_state(self._h, _ptr(p), _ptr(m), _ptr(v), C.byref(count), _stream()))
        return p, m, v, int(count.value)

    def load_state(self, params: torch.Tensor, mu: torch.Tensor | None = None,
                   nu: torch.Tensor | None = None, count: torch.Tensor | None = None):
        """Stream-ordered device copies of a flat state into the handle (no host
        synchronisation); count is an int32 device scalar. None leaves a part as it is."""
        cnt = None
        if count is not None:
            cnt = count.to(self.device, torch.int32).reshape(1).contiguous()
        _lib.check(_lib.lib().bt_learner_load_state(
            self._h, _ptr(params.contiguous()), _ptr(mu.contiguous()) if mu is not None else None,
            _ptr(nu.contiguous()) if nu is not None else None, _ptr(cnt), _stream()))
        return cnt  # keeps the source of the asynchronous copy alive for the caller

    def store_state(self):
        """The handle's state as new device tensors (params, mu, nu, count [int32 scalar]),
        copied on the current stream without a host synchronisation."""
        p = torch.empty(self.num_params, dtype=torch.float32, device=self.device)
        m, v = torch.empty_like(p), torch.empty_like(p)
        c = torch.empty((), dtype=torch.int32, device=self.device)
        _lib.check(_lib.lib().bt_learner_store_state(self._h, _ptr(p), _ptr(m), _ptr(v), _ptr(c),
                                                     _stream()))
        return p, m, v, c

    def params(self) -> dict:
        p, _, _, _ = self.get_state()
        return self.layout.unflatten(p.cpu().numpy())

    # ---- compute -----------------------------------------------------------------------------
    def _batch(self, batch: dict) -> _lib.Batch:
        b = _lib.Batch()
        for f in BATCH_FIELDS:
            t = batch.get(f)
            setattr(b, f, _ptr(t) if t is not None else None)
        return b

    def update(self, batch: dict, permutations: torch.Tensor, stats: bool = True):
        b = self._batch(batch)
        st = None
        if stats:
            st = torch.empty(self.ppo.update_epochs, self.ppo.num_minibatches, _lib.NUM_STATS,
                             dtype=torch.float32, device=self.device)
        perm = permutations.to(self.device, torch.int32).contiguous()
        _lib.check(_lib.lib().bt_learner_update(self._h, C.byref(b), _ptr(perm), _ptr(st), _stream()))
        return st

    def check(self):
        """Synchronise and raise if a kernel of an earlier call recorded a failure."""
        _lib.check(_lib.lib().bt_learner_check(self._h, _stream()))

    def use_graphs(self, enable: bool = True):
        """Replay updates as a captured CUDA graph (the default) or enqueue them eagerly."""
        _lib.check(_lib.lib().bt_learner_use_graphs(self._h, int(enable)))

    def targets(self):
        n = self.num_steps * self.num_envs
        adv = torch.empty(n, dtype=torch.float32, device=self.device)
        ret, boot = torch.empty_like(adv), torch.empty(self.num_envs, dtype=torch.float32, device=self.device)
        _lib.check(_lib.lib().bt_learner_targets(self._h, _ptr(adv), _ptr(ret), _ptr(boot), _stream()))
        return adv, ret, boot

    def loss_grads(self, batch: dict, advantages, returns, indices):
        b = self._batch(batch)
        idx = indices.to(self.device, torch.int32).contiguous()
        g = torch.empty(self.num_params, dtype=torch.float32, device=self.device)
        st = torch.empty(_lib.NUM_STATS, dtype=torch.float32, device=self.device)
        _lib.check(_lib.lib().bt_learner_loss_grads(
            self._h, C.byref(b), _ptr(advantages.contiguous()), _ptr(returns.contiguous()),
            _ptr(idx), int(idx.numel()), _ptr(g), _ptr(st), _stream()))
        return g, st

    def act(self, obs: torch.Tensor, noise: torch.Tensor | None = None, temperature: float = 1.0):
        num = obs.shape[0]
        a = self.network.action_dim
        if self.network.head == "categorical":
            action = torch.empty(num, dtype=torch.int32, device=self.device)
        else:
            action = torch.empty(num, a, dtype=torch.float32, device=self.device)
        lp = torch.empty(num, dtype=torch.float32, device=self.device)
        value = torch.empty(num, dtype=torch.float32, device=self.device)
        _lib.check(_lib.lib().bt_learner_act(
            self._h, _ptr(obs.contiguous()), num, _ptr(noise.contiguous()) if noise is not None else None,
            float(temperature), _ptr(action), _ptr(lp), _ptr(value), _stream()))
        return action, lp, value

    def act_recurrent(self, obs: torch.Tensor, reset: torch.Tensor, carry: torch.Tensor,
                      noise: torch.Tensor | None = None, temperature: float = 1.0):
        """One step of a GRU network (RecurrentPPO.step): obs [num, D], reset [num] (the carry
        is zeroed where set), carry [num, H]. Returns (action, log_prob, value, new carry)."""
        num = obs.shape[0]
        a = self.network.action_dim
        if self.network.head == "categorical":
            action = torch.empty(num, dtype=torch.int32, device=self.device)
        else:
            action = torch.empty(num, a, dtype=torch.float32, device=self.device)
        lp = torch.empty(num, dtype=torch.float32, device=self.device)
        value = torch.empty(num, dtype=torch.float32, device=self.device)
        new_carry = torch.empty_like(carry, dtype=torch.float32)
        _lib.check(_lib.lib().bt_learner_act_recurrent(
            self._h, _ptr(obs.contiguous()), _ptr(reset.to(torch.uint8).contiguous()),
            _ptr(carry.to(torch.float32).contiguous()), num,
            _ptr(noise.contiguous()) if noise is not None else None, float(temperature),
            _ptr(action), _ptr(lp), _ptr(value), _ptr(new_carry), _stream()))
        return action, lp, value, new_carry

    # ---- tracing -------------------------------------------------------------------------------
    def profile(self, enable: bool = True):
        _lib.check(_lib.lib().bt_learner_profile(self._h, int(enable)))

    def profile_read(self) -> dict:
        """{kernel class: (total device ms, launches)} of the recorded launches."""
        L = _lib.lib()
        out = {}
        name = C.create_string_buffer(64)
        ms, n = C.c_double(), C.c_int64()
        cls = 0
        while L.bt_learner_profile_read(self._h, cls, name, 64, C.byref(ms), C.byref(n)) == 0:
            if n.value:
                out[name.value.decode()] = (ms.value, n.value)
            cls += 1
        return out

    def launch_count(self) -> int:
        return int(_lib.lib().bt_learner_launch_count(self._h))

    # ---- multi-GPU -----------------------------------------------------------------------------
    @staticmethod
    def nccl_unique_id() -> bytes:
        buf = C.create_string_buffer(128)
        _lib.check(_lib.lib().bt_nccl_unique_id(buf, 128))
        return buf.raw

    def comm_init(self, unique_id: bytes):
        buf = C.create_string_buffer(bytes(unique_id), 128)
        _lib.check(_lib.lib().bt_learner_comm_init(self._h, buf, 128))

    def use_p2p(self, enable: bool = True):
        """The NVLink peer-memory gradient exchange fused with the optimizer step (default
        when available), or the NCCL all-reduce with the full optimizer step (False)."""
        _lib.check(_lib.lib().bt_learner_use_p2p(self._h, int(enable)))


def gae(reward, terminated, truncated, values, bootstrap, gamma: float, gae_lambda: float,
        rho=None, c=None):
    """generalized_advantage_estimator (boonta/algorithms/advantage_estimators.py:8-56) on
    CUDA tensors [T, N]; returns (advantages, returns)."""
    t, n = reward.shape
    adv = torch.empty((t, n), dtype=torch.float32, device=reward.device)
    ret = torch.empty_like(adv)
    _lib.check(_lib.lib().bt_gae(
        _ptr(reward.contiguous()), _ptr(terminated.contiguous()), _ptr(truncated.contiguous()),
        _ptr(values.contiguous()), _ptr(bootstrap.contiguous()),
        _ptr(rho.contiguous()) if rho is not None else None,
        _ptr(c.contiguous()) if c is not None else None,
        t, n, float(gamma), float(gae_lambda), _ptr(adv), _ptr(ret), _stream()))
    return adv, ret


def sample_categorical(logits: torch.Tensor, uniforms: torch.Tensor | None, temperature: float = 1.0):
    rows, a = logits.shape
    action = torch.empty(rows, dtype=torch.int32, device=logits.device)
    lp = torch.empty(rows, dtype=torch.float32, device=logits.device)
    _lib.check(_lib.lib().bt_sample_categorical(
        _ptr(logits.contiguous()), _ptr(uniforms.contiguous()) if uniforms is not None else None,
        rows, a, float(temperature), _ptr(action), _ptr(lp), _stream()))
    return action, lp


def to_device(rollout: dict, device="cuda") -> dict:
    """numpy rollout (boonta_b200.configs.rollout) -> CUDA tensors with the C-ABI dtypes."""
    out = {}
    for k, v in rollout.items():
        t = torch.from_numpy(np.ascontiguousarray(v))
        if t.dtype == torch.bool:
            t = t.to(torch.uint8)
        out[k] = t.to(device)
    return out
