"""ctypes binding of the C-ABI in include/boonta_b200.h.

This is the same binding a JAX host would hold next to its jax.ffi registration (the
reference registers its native targets through ctypes + jax.ffi in
boonta/environments/__init__.py:10-43). The library is built in-tree
(`python -m boonta_b200.build`); importing this module without it raises, so there is no
silent fallback path.
"""
from __future__ import annotations

import ctypes as C
from pathlib import Path

LIB_PATH = Path(__file__).resolve().parent / "libboonta_b200.so"

BT_OK = 0
BT_ERR_INVALID = -1
BT_ERR_CUDA = -2
BT_ERR_NCCL = -3
BT_ERR_TIMEOUT = -4
BT_ERR_CAPACITY = -5
BT_ERR_UNSUPPORTED = -6

BT_LAYER_DENSE, BT_LAYER_CONV3X3, BT_LAYER_GRU = 0, 1, 2
ACT = {"none": 0, "tanh": 1, "relu": 2, "silu": 3}
HEAD = {"categorical": 0, "gaussian": 1}
PRECISION = {"fp32": 0, "bf16": 1, "bf16x3": 2}
MAX_LAYERS = 8
NUM_STATS = 8

# Every function the header declares (checked against the built library by the tests).
EXPORTS = (
    "bt_last_error", "bt_version", "bt_gae", "bt_learner_create", "bt_learner_destroy",
    "bt_learner_num_params", "bt_learner_param_count", "bt_learner_param_info",
    "bt_learner_set_state", "bt_learner_get_state", "bt_learner_update", "bt_learner_targets",
    "bt_learner_loss_grads", "bt_learner_act", "bt_learner_act_recurrent",
    "bt_sample_categorical", "bt_nccl_unique_id",
    "bt_learner_comm_init", "bt_learner_profile", "bt_learner_profile_read",
    "bt_learner_launch_count", "bt_gemm_bf16", "bt_gemm_bf16x3", "bt_clip_adam",
    "bt_clip_adam_noalloc", "bt_learner_use_graphs", "bt_learner_check",
    "bt_selftest_bounded_wait", "bt_learner_load_state", "bt_learner_store_state",
    "bt_learner_use_p2p", "bt_learner_exchange_probe", "bt_linear_scan",
    "bt_linear_scan_backward", "bt_threefry2x32_host", "bt_threefry2x32", "bt_random_split",
    "bt_random_fill", "bt_random_permutation_workspace", "bt_random_permutation",
    "bt_selftest_gru_barrier",
)


class Layer(C.Structure):
    _fields_ = [
        ("kind", C.c_int32), ("features", C.c_int32), ("activation", C.c_int32),
        ("layernorm", C.c_int32), ("height", C.c_int32), ("width", C.c_int32),
        ("in_channels", C.c_int32),
    ]


class Network(C.Structure):
    _fields_ = [
        ("obs_dim", C.c_int32), ("num_torso", C.c_int32), ("torso", Layer * MAX_LAYERS),
        ("num_critic", C.c_int32), ("critic", Layer * MAX_LAYERS), ("head", C.c_int32),
        ("action_dim", C.c_int32),
    ]


class PPOConfigC(C.Structure):
    _fields_ = [
        ("num_minibatches", C.c_int32), ("update_epochs", C.c_int32),
        ("clip_coefficient", C.c_float), ("clip_value_loss", C.c_int32),
        ("entropy_coefficient", C.c_float), ("value_coefficient", C.c_float),
        ("gamma", C.c_double), ("gae_lambda", C.c_double), ("normalize_advantage", C.c_int32),
    ]


class OptimizerC(C.Structure):
    _fields_ = [(n, C.c_float) for n in ("lr", "max_grad_norm", "b1", "b2", "eps", "eps_root")]


class LearnerConfig(C.Structure):
    _fields_ = [
        ("network", Network), ("ppo", PPOConfigC), ("optimizer", OptimizerC),
        ("num_steps", C.c_int32), ("num_envs", C.c_int32), ("precision", C.c_int32),
        ("world_size", C.c_int32), ("rank", C.c_int32),
    ]


class Batch(C.Structure):
    _fields_ = [
        ("obs", C.c_void_p), ("bootstrap_obs", C.c_void_p), ("action", C.c_void_p),
        ("reward", C.c_void_p), ("terminated", C.c_void_p), ("truncated", C.c_void_p),
        ("log_prob", C.c_void_p), ("value", C.c_void_p), ("first_done", C.c_void_p),
        ("carry", C.c_void_p), ("last_carry", C.c_void_p),
    ]


class BoontaError(RuntimeError):
    def __init__(self, code: int, message: str):
        super().__init__(f"[{code}] {message}")
        self.code = code


_lib = None


def lib() -> C.CDLL:
    global _lib
    if _lib is not None:
        return _lib
    if not LIB_PATH.exists():
        raise ImportError(
            f"{LIB_PATH} is missing: build it with `python -m boonta_b200.build` "
            "(the CUDA library has no CPU fallback)"
        )
    L = C.CDLL(str(LIB_PATH))
    vp, i32, i64, f32, f64 = C.c_void_p, C.c_int32, C.c_int64, C.c_float, C.c_double
    sig = {
        "bt_last_error": (C.c_char_p, []),
        "bt_version": (C.c_char_p, []),
        "bt_gae": (C.c_int, [vp, vp, vp, vp, vp, vp, vp, i32, i32, f64, f64, vp, vp, vp]),
        "bt_linear_scan": (C.c_int, [vp, vp, vp, vp, i32, i32, i32, i32, i32, vp]),
        "bt_selftest_gru_barrier": (C.c_int, [i32, vp]),
        "bt_threefry2x32_host": (None, [C.c_uint32, C.c_uint32, C.c_uint32, C.c_uint32,
                                        C.POINTER(C.c_uint32)]),
        "bt_threefry2x32": (C.c_int, [C.c_uint32, C.c_uint32, vp, vp, vp, vp, i64, vp]),
        "bt_random_split": (C.c_int, [C.POINTER(C.c_uint32), i32, i32, C.POINTER(C.c_uint32)]),
        "bt_random_fill": (C.c_int, [C.POINTER(C.c_uint32), i64, i32, C.c_float, C.c_float, i32,
                                     vp, vp]),
        "bt_random_permutation_workspace": (i64, [i64]),
        "bt_random_permutation": (C.c_int, [C.POINTER(C.c_uint32), i64, i32, vp, vp, i64, vp]),
        "bt_linear_scan_backward": (C.c_int, [vp, vp, vp, vp, vp, vp, vp, i32, i32, i32, i32,
                                              i32, vp]),
        "bt_learner_create": (C.c_int, [C.POINTER(LearnerConfig), C.POINTER(vp)]),
        "bt_learner_destroy": (None, [vp]),
        "bt_learner_num_params": (i64, [vp]),
        "bt_learner_param_count": (i32, [vp]),
        "bt_learner_param_info": (C.c_int, [vp, i32, C.c_char_p, i32, C.POINTER(i64),
                                            C.POINTER(i32), C.POINTER(i64)]),
        "bt_learner_set_state": (C.c_int, [vp, vp, vp, vp, i32, vp]),
        "bt_learner_get_state": (C.c_int, [vp, vp, vp, vp, C.POINTER(i32), vp]),
        "bt_learner_load_state": (C.c_int, [vp, vp, vp, vp, vp, vp]),
        "bt_learner_store_state": (C.c_int, [vp, vp, vp, vp, vp, vp]),
        "bt_learner_update": (C.c_int, [vp, C.POINTER(Batch), vp, vp, vp]),
        "bt_learner_use_graphs": (C.c_int, [vp, i32]),
        "bt_learner_check": (C.c_int, [vp, vp]),
        "bt_selftest_bounded_wait": (C.c_int, [i32, vp]),
        "bt_learner_targets": (C.c_int, [vp, vp, vp, vp, vp]),
        "bt_learner_loss_grads": (C.c_int, [vp, C.POINTER(Batch), vp, vp, vp, i32, vp, vp, vp]),
        "bt_learner_act": (C.c_int, [vp, vp, i32, vp, f32, vp, vp, vp, vp]),
        "bt_learner_act_recurrent": (C.c_int, [vp, vp, vp, vp, i32, vp, f32, vp, vp, vp, vp,
                                               vp]),
        "bt_sample_categorical": (C.c_int, [vp, vp, i32, i32, f32, vp, vp, vp]),
        "bt_nccl_unique_id": (C.c_int, [vp, i32]),
        "bt_learner_comm_init": (C.c_int, [vp, vp, i32]),
        "bt_learner_use_p2p": (C.c_int, [vp, i32]),
        "bt_learner_exchange_probe": (C.c_int, [vp, i32, i32, vp]),
        "bt_learner_profile": (C.c_int, [vp, i32]),
        "bt_learner_profile_read": (C.c_int, [vp, i32, C.c_char_p, i32, C.POINTER(f64),
                                              C.POINTER(i64)]),
        "bt_learner_launch_count": (i64, [vp]),
        "bt_gemm_bf16": (C.c_int, [vp, vp, vp, i32, i32, i32, i32, i32, i32, vp, vp]),
        "bt_gemm_bf16x3": (C.c_int, [vp, vp, vp, vp, vp, i32, i32, i32, i32, i32, vp]),
        "bt_clip_adam": (C.c_int, [vp, vp, vp, vp, i64, i32, C.POINTER(OptimizerC), vp]),
        "bt_clip_adam_noalloc": (C.c_int, [vp, vp, vp, vp, i64, i32, C.POINTER(OptimizerC), vp]),
    }
    for name, (res, args) in sig.items():
        fn = getattr(L, name)
        fn.restype = res
        fn.argtypes = args
    _lib = L
    return L


def check(code: int) -> None:
    if code != BT_OK:
        raise BoontaError(code, lib().bt_last_error().decode(errors="replace"))
