"""jax.ffi binding of the learner path (needs jax and a library built with JAXLIB_INCLUDE).

The reference registers native code with JAX as XLA FFI targets: the handler pointer from an
extern "C" getter, wrapped in a PyCapsule, passed to jax.ffi.register_ffi_target
(boonta/environments/__init__.py:10-15, 38-43). This module does the same for the learner's
handlers (boonta_b200/csrc/xla_ffi.cc) and gives the calls a JAX host makes in place of
boonta's PPO.update / PPO.step / generalized_advantage_estimator:

    from boonta_b200 import jax_ffi
    jax_ffi.register()
    adv, ret = jax_ffi.gae(reward, terminated, truncated, values, bootstrap, gamma, lam)
    state, stats = jax_ffi.ppo_update(learner, state, transitions, permutations)

`learner` is a boonta_b200.learner.Learner created once per device (its handle is the
"learner" attribute of the custom call); the functional state is (params, mu, nu, count) as
flat float32 arrays in the learner's layout plus an int32 scalar. jax is not installed in this
image, so this module is not exercised by the test suite here.
"""
from __future__ import annotations

import ctypes

import numpy as np

from . import _lib

TARGETS = {
    "boonta_gae": "bt_xla_gae_handler",
    "boonta_ppo_update": "bt_xla_ppo_update_handler",
    "boonta_recurrent_ppo_update": "bt_xla_recurrent_ppo_update_handler",
    "boonta_ppo_act": "bt_xla_ppo_act_handler",
}

_registered = False


def _capsule(address: int):
    new = ctypes.pythonapi.PyCapsule_New
    new.restype = ctypes.py_object
    new.argtypes = [ctypes.c_void_p, ctypes.c_char_p, ctypes.c_void_p]
    return new(address, None, None)


def register() -> None:
    """Registers the four handlers for the CUDA platform (once per process)."""
    global _registered
    if _registered:
        return
    import jax

    lib = _lib.lib()
    for name, getter in TARGETS.items():
        if not hasattr(lib, getter):
            raise RuntimeError(
                f"{_lib.LIB_PATH} has no {getter}: rebuild with JAXLIB_INCLUDE set to "
                "jax.ffi.include_dir()")
        fn = getattr(lib, getter)
        fn.restype = ctypes.c_void_p
        jax.ffi.register_ffi_target(name, _capsule(fn()), platform="CUDA")
    _registered = True


def gae(reward, terminated, truncated, values, bootstrap, gamma: float, gae_lambda: float):
    """generalized_advantage_estimator (advantage_estimators.py:8-56) on [T, N] arrays."""
    import jax
    import jax.numpy as jnp

    out = jax.ShapeDtypeStruct(reward.shape, jnp.float32)
    return jax.ffi.ffi_call("boonta_gae", (out, out))(
        reward, terminated.astype(jnp.bool_), truncated.astype(jnp.bool_), values, bootstrap,
        gamma=np.float64(gamma), gae_lambda=np.float64(gae_lambda))


def ppo_update(learner, state, transitions: dict, permutations):
    """One PPO.update (ppo.py:76-233) as a pure function of state = (params, mu, nu, count).
    transitions: first.obs, second.obs[-1], second.action / reward / terminated / truncated,
    aux.log_prob / value as the dict keys of boonta_b200.learner.BATCH_FIELDS (plus first_done,
    carry, last_carry for GRU networks); permutations: int32 [E, T*N*world] (or [E, N*world]
    environment permutations for GRU networks). Returns (new state, stats [E, M, 8])."""
    import jax
    import jax.numpy as jnp

    params, mu, nu, count = state
    e, m = learner.ppo.update_epochs, learner.ppo.num_minibatches
    outs = (jax.ShapeDtypeStruct(params.shape, jnp.float32),) * 3 + (
        jax.ShapeDtypeStruct((), jnp.int32), jax.ShapeDtypeStruct((e, m, _lib.NUM_STATS),
                                                                  jnp.float32))
    t = transitions
    args = [t["obs"], t["bootstrap_obs"], t["action"], t["reward"],
            t["terminated"].astype(jnp.bool_), t["truncated"].astype(jnp.bool_), t["log_prob"],
            t["value"]]
    target = "boonta_ppo_update"
    if learner.network.recurrent:
        target = "boonta_recurrent_ppo_update"
        args += [t["first_done"].astype(jnp.bool_), t["carry"], t["last_carry"]]
    args += [permutations.astype(jnp.int32), params, mu, nu, jnp.asarray(count, jnp.int32)]
    p, m_, v, c, stats = jax.ffi.ffi_call(target, outs)(*args, learner=np.int64(learner.handle))
    return (p, m_, v, c), stats


def ppo_act(learner, params, obs, noise=None, temperature: float = 1.0):
    """PPO.step (ppo.py:57-74): (action, log_prob, value) for obs [num, obs_dim]."""
    import jax
    import jax.numpy as jnp

    num = obs.shape[0]
    a = learner.network.action_dim
    action = (jax.ShapeDtypeStruct((num,), jnp.int32) if learner.network.head == "categorical"
              else jax.ShapeDtypeStruct((num, a), jnp.float32))
    noise = jnp.zeros((0,), jnp.float32) if noise is None else noise
    outs = (action, jax.ShapeDtypeStruct((num,), jnp.float32),
            jax.ShapeDtypeStruct((num,), jnp.float32))
    return jax.ffi.ffi_call("boonta_ppo_act", outs)(
        obs, noise, params, learner=np.int64(learner.handle), temperature=np.float32(temperature))
