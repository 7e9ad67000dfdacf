"""PPOState as the reference's pytree, and a checkpoint file of it.

boonta's PPOState is `PPOState(step, params, optimizer_state)` (boonta/algorithms/ppo.py:30-34)
with the optax chain state of `optax.chain(clip_by_global_norm, adam)`: the tuple
`(EmptyState(), ScaleByAdamState(count, mu, nu), EmptyState())` whose mu and nu mirror the
params tree. Checkpoints hold that tree, either as orbax directories
(boonta/loggers/orbax.py:55-75) or as one flax-serialised msgpack file
(boonta/utils/checkpoint.py:122-127: `serialization.msgpack_restore` / `from_bytes`).

Here the learner keeps params, mu and nu as flat buffers (boonta_b200.spec.param_layout).
`state_pytree` maps a PPOState to the reference's tree shape (params nested by the layout's
"/"-separated names; the optax chain as a 3-tuple with the adam state in the middle), and
`save` / `load` write and read it in flax's msgpack state-dict encoding: namedtuples and tuples
become maps (tuple positions keyed "0", "1", "2"), arrays msgpack extension type 1 holding
(shape, dtype name, C-order bytes), numpy scalars extension type 3 (dtype name, bytes). orbax is
not installed here, so the directory format is not written. The parameter names are this
library's (a flax module names its own), so the tree's layout, not its leaf names, is what
carries over.
"""
from __future__ import annotations

from collections import namedtuple
from pathlib import Path

import msgpack
import numpy as np

EmptyState = namedtuple("EmptyState", [])
ScaleByAdamState = namedtuple("ScaleByAdamState", ["count", "mu", "nu"])

_EXT_NDARRAY = 1
_EXT_NPSCALAR = 3


def _nest(layout, flat: np.ndarray) -> dict:
    tree: dict = {}
    for e in layout.entries:
        node = tree
        parts = e.name.split("/")
        for p in parts[:-1]:
            node = node.setdefault(p, {})
        n = int(np.prod(e.shape)) if e.shape else 1
        node[parts[-1]] = np.asarray(flat[e.offset:e.offset + n], np.float32).reshape(e.shape)
    return tree


def _unnest(layout, tree: dict) -> np.ndarray:
    flat = np.zeros(layout.total, np.float32)
    for e in layout.entries:
        node = tree
        for p in e.name.split("/"):
            node = node[p]
        n = int(np.prod(e.shape)) if e.shape else 1
        flat[e.offset:e.offset + n] = np.asarray(node, np.float32).reshape(-1)
    return flat


def _host(x) -> np.ndarray:
    try:
        import torch

        if isinstance(x, torch.Tensor):
            return x.detach().cpu().numpy()
    except ImportError:
        pass
    return np.asarray(x)


def state_pytree(state, layout) -> dict:
    """The reference's PPOState tree of a boonta_b200.ppo.PPOState (host numpy leaves):
    {"step", "params", "optimizer_state": (EmptyState(), ScaleByAdamState(count, mu, nu),
    EmptyState())}."""
    opt = state.optimizer_state
    return {
        "step": np.int64(_host(state.step)),
        "params": _nest(layout, _host(state.params).reshape(-1)),
        "optimizer_state": (EmptyState(),
                            ScaleByAdamState(count=np.int32(_host(opt.count)),
                                             mu=_nest(layout, _host(opt.mu).reshape(-1)),
                                             nu=_nest(layout, _host(opt.nu).reshape(-1))),
                            EmptyState()),
    }


def from_state_pytree(tree: dict, layout, device="cuda"):
    """The boonta_b200.ppo.PPOState of a tree from state_pytree (or from load)."""
    import torch

    from .ppo import AdamState, PPOState

    chain = tree["optimizer_state"]
    adam = chain[1] if isinstance(chain, (tuple, list)) else chain["1"]
    if isinstance(adam, dict):
        adam = ScaleByAdamState(adam["count"], adam["mu"], adam["nu"])
    flat = lambda t: torch.as_tensor(_unnest(layout, t), device=device)
    return PPOState(step=torch.tensor(int(tree["step"]), dtype=torch.int64),
                    params=flat(tree["params"]),
                    optimizer_state=AdamState(flat(adam.mu), flat(adam.nu),
                                              torch.tensor(int(adam.count), dtype=torch.int32,
                                                           device=device)))


def to_state_dict(x):
    """flax.serialization.to_state_dict for the tree's node types: dicts, tuples (keys "0",
    "1", ...), namedtuples (their field names)."""
    if isinstance(x, dict):
        return {str(k): to_state_dict(v) for k, v in x.items()}
    if isinstance(x, tuple) and hasattr(x, "_fields"):
        return {f: to_state_dict(getattr(x, f)) for f in x._fields}
    if isinstance(x, (tuple, list)):
        return {str(i): to_state_dict(v) for i, v in enumerate(x)}
    return x


def _encode(obj):
    if isinstance(obj, np.ndarray):
        return msgpack.ExtType(_EXT_NDARRAY, msgpack.packb(
            (obj.shape, obj.dtype.name, np.ascontiguousarray(obj).tobytes()), use_bin_type=True))
    if isinstance(obj, np.generic):
        return msgpack.ExtType(_EXT_NPSCALAR, msgpack.packb(
            (obj.dtype.name, obj.tobytes()), use_bin_type=True))
    raise TypeError(f"cannot serialise {type(obj).__name__}")


def _decode(code, data):
    if code == _EXT_NDARRAY:
        shape, dtype, buf = msgpack.unpackb(data, raw=False)
        return np.frombuffer(buf, dtype=np.dtype(dtype)).reshape(shape).copy()
    if code == _EXT_NPSCALAR:
        dtype, buf = msgpack.unpackb(data, raw=False)
        return np.frombuffer(buf, dtype=np.dtype(dtype))[0]
    return msgpack.ExtType(code, data)


def to_bytes(state, layout) -> bytes:
    """The state's tree in flax's msgpack state-dict encoding."""
    return msgpack.packb(to_state_dict(state_pytree(state, layout)), default=_encode,
                         use_bin_type=True)


def from_bytes(data: bytes) -> dict:
    """The state-dict tree of to_bytes (maps with string keys; numpy leaves)."""
    return msgpack.unpackb(data, ext_hook=_decode, raw=False, strict_map_key=False)


def save(path, state, layout) -> Path:
    path = Path(path)
    path.write_bytes(to_bytes(state, layout))
    return path


def load(path, layout, device="cuda"):
    """The PPOState saved by `save`."""
    return from_state_pytree(from_bytes(Path(path).read_bytes()), layout, device)
