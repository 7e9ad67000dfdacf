"""Host-side statement of how a global minibatch splits across ranks (data parallelism over
the env axis, boonta/podracers/anakin.py:165-186).

The reference permutes the *global* batch (boonta/algorithms/ppo.py:200), so a minibatch
is a set of global flat indices i = t * N_global + n_global. Rank r owns envs
[r*N, (r+1)*N); its rows of the minibatch are the owned indices, in permutation order,
mapped to local flat indices t * N + (n_global - r*N). The CUDA learner does the same on
the device (local_indices_kernel); this numpy version documents the rule and drives the
multi-process CPU tests.
"""
from __future__ import annotations

import numpy as np


def local_rows(global_indices: np.ndarray, rank: int, n_local: int, world: int) -> np.ndarray:
    g = np.asarray(global_indices, np.int64)
    n_global = n_local * world
    t, ng = np.divmod(g, n_global)
    mine = (ng // n_local) == rank
    return (t[mine] * n_local + (ng[mine] - rank * n_local)).astype(np.int32)
