"""The SSM torso's linear recurrence h_t = a_t h_{t-1} + b_t and its custom VJP, restated from
boonta/networks/kernels/scan.py (test infrastructure only).

* `sequential`: the reference's `_forward` (:13-38) / `sequential` (:119-131) order, a float32
  carry from init over the steps, stored in a's dtype (float32, or bfloat16 as float32 values
  rounded with `bf16_round`).
* `backward`: `_backward` (:41-68) and `_scan_bwd` (:81-87): g_{T-1} = cot_{T-1},
  g_t = cot_t + a_{t+1} g_{t+1} in float32 after casting the cotangent to a's dtype; db = g in
  a's dtype; da = db * concat(init, h[:, :-1]) (the concatenation takes the promoted dtype, so
  an fp32 init enters unrounded) rounded to a's dtype; dinit = (db[:, 0] * a[:, 0]) in a's
  dtype, then init's dtype.
* `exact`: float64 evaluation of the recurrence (the `associative` reference of the reference's
  tests, without rounding).
* `chunked` / `chunked_backward`: the CUDA kernels' evaluation order (boonta_b200/csrc/scan.cu):
  the steps in 8 chunks of ceil(T / 8); each chunk folded into an affine map from a zero carry,
  the maps composed in order onto the initial carry, then each chunk rescanned; every product
  and sum rounded to float32 separately. Bit-identical to the kernels.
"""
from __future__ import annotations

import numpy as np

from .network import bf16_round

CHUNKS = 8


def _store(x, bf16: bool):
    x = np.asarray(x, np.float32)
    return bf16_round(x) if bf16 else x


def _f32(x):
    return np.asarray(x, np.float32)


def exact(a, b, init):
    a, b, init = (np.asarray(x, np.float64) for x in (a, b, init))
    out = np.empty_like(a)
    h = init
    for t in range(a.shape[1]):
        h = a[:, t] * h + b[:, t]
        out[:, t] = h
    return out


def sequential(a, b, init, bf16: bool = False):
    a, b, h = _f32(a), _f32(b), _f32(init).copy()
    out = np.empty_like(a)
    for t in range(a.shape[1]):
        h = (a[:, t] * h + b[:, t]).astype(np.float32)
        out[:, t] = _store(h, bf16)
    return out


def backward(a, h, init, cot, bf16: bool = False):
    """(da, db, dinit) of the reference's custom VJP, sequential order."""
    a, h, init = _f32(a), _f32(h), _f32(init)
    cot = _store(cot, bf16)
    T = a.shape[1]
    db = np.empty_like(a)
    g = cot[:, T - 1].copy()
    db[:, T - 1] = _store(g, bf16)
    for t in range(T - 2, -1, -1):
        g = (cot[:, t] + (a[:, t + 1] * g).astype(np.float32)).astype(np.float32)
        db[:, t] = _store(g, bf16)
    shifted = np.concatenate([init[:, None], h[:, :-1]], axis=1)
    da = _store(db * shifted, bf16)
    dinit = _store(db[:, 0] * a[:, 0], bf16)
    return da, db, dinit


def _chunks(T):
    L = -(-T // CHUNKS)
    return [(min(T, w * L), min(T, w * L + L)) for w in range(CHUNKS)]


def chunked(a, b, init, bf16: bool = False):
    a, b = _f32(a), _f32(b)
    T = a.shape[1]
    spans = _chunks(T)
    maps = []
    for t0, t1 in spans:
        m = np.ones(a.shape[0::2], np.float32)
        c = np.zeros(a.shape[0::2], np.float32)
        for t in range(t0, t1):
            m = (a[:, t] * m).astype(np.float32)
            c = ((a[:, t] * c).astype(np.float32) + b[:, t]).astype(np.float32)
        maps.append((m, c))
    out = np.empty_like(a)
    for w, (t0, t1) in enumerate(spans):
        h = _f32(init).copy()
        for k in range(w):
            m, c = maps[k]
            h = ((m * h).astype(np.float32) + c).astype(np.float32)
        for t in range(t0, t1):
            h = ((a[:, t] * h).astype(np.float32) + b[:, t]).astype(np.float32)
            out[:, t] = _store(h, bf16)
    return out


def chunked_backward(a, h, init, cot, bf16: bool = False):
    a, h, init = _f32(a), _f32(h), _f32(init)
    cot = _store(cot, bf16)
    T = a.shape[1]
    spans = _chunks(T)

    def mult(t):
        return a[:, t + 1] if t + 1 < T else np.zeros(a.shape[0::2], np.float32)

    maps = []
    for t0, t1 in spans:
        m = np.ones(a.shape[0::2], np.float32)
        c = np.zeros(a.shape[0::2], np.float32)
        for t in range(t1 - 1, t0 - 1, -1):
            mt = mult(t)
            m = (mt * m).astype(np.float32)
            c = ((mt * c).astype(np.float32) + cot[:, t]).astype(np.float32)
        maps.append((m, c))
    da = np.empty_like(a)
    db = np.empty_like(a)
    dinit = None
    for w, (t0, t1) in enumerate(spans):
        g = np.zeros(a.shape[0::2], np.float32)
        for k in range(CHUNKS - 1, w, -1):
            m, c = maps[k]
            g = ((m * g).astype(np.float32) + c).astype(np.float32)
        for t in range(t1 - 1, t0 - 1, -1):
            g = ((mult(t) * g).astype(np.float32) + cot[:, t]).astype(np.float32)
            gs = _store(g, bf16)
            db[:, t] = gs
            hp = h[:, t - 1] if t > 0 else init
            da[:, t] = _store((gs * hp).astype(np.float32), bf16)
            if t == 0:
                dinit = _store((gs * a[:, 0]).astype(np.float32), bf16)
    return da, db, dinit
