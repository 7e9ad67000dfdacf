"""boonta_b200: a B200-native (sm_100a) implementation of boonta's Anakin PPO learner step.

The compute lives in the CUDA library `libboonta_b200.so` (C-ABI: include/boonta_b200.h);
this package holds the host side: the network/algorithm specifications (`spec`), the
synthetic workloads (`configs`), the ctypes binding (`_lib`), the learner handle
(`learner.Learner`) and the boonta-compatible `PPO` class (`ppo`).
"""
from .spec import (GRU, Conv3x3, Dense, NetworkSpec, OptimizerConfig, PPOConfig,  # noqa: F401
                   param_layout)

__version__ = "0.1.0"


def __getattr__(name):
    if name in ("Learner", "gae", "sample_categorical"):
        from . import learner

        return getattr(learner, name)
    if name in ("PPO", "PPOState", "RecurrentPPO", "RecurrentPPOState", "RecurrentPPOConfig",
                "Timestep", "Transition", "AdamState", "generalized_advantage_estimator"):
        from . import ppo

        return getattr(ppo, name)
    raise AttributeError(name)
