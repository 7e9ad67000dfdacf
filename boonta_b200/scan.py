"""The SSM torso's linear recurrence on the GPU (boonta/networks/kernels/scan.py).

`scan(a, b, init)` is the reference's `scan` (a custom-VJP function, :71-89) on CUDA tensors:
h[:, t] = a[:, t] * h[:, t-1] + b[:, t] from h[:, -1] = init over [batch, steps, features]
(extra feature axes are folded like the reference's `pallas` wrapper, :92-103), accumulated in
float32 and returned in a's dtype (float32 or bfloat16), differentiable through the native
backward kernel. `get_scan_implementation` mirrors the reference's registry
(boonta/networks/kernels/__init__.py:12-19) with the native kernel under "cuda" (the default,
the role "pallas" plays there) and the two pure-torch forms for comparison.
"""
from __future__ import annotations

import torch

from . import _lib

_DTYPES = {torch.float32: 0, torch.bfloat16: 1}


def _ptr(t: torch.Tensor):
    return t.data_ptr() if t.numel() else None


def _stream():
    return torch.cuda.current_stream().cuda_stream


def _check(a, b, init):
    if not (a.is_cuda and b.is_cuda and init.is_cuda):
        raise ValueError("scan: CUDA tensors expected")
    if a.dtype not in _DTYPES or init.dtype not in _DTYPES:
        raise TypeError(f"scan: dtypes {a.dtype} / {init.dtype} (float32 or bfloat16 expected)")
    if a.shape != b.shape or a.ndim != 3 or init.shape != (a.shape[0], a.shape[2]):
        raise ValueError(f"scan: shapes a {tuple(a.shape)}, b {tuple(b.shape)}, "
                         f"init {tuple(init.shape)}")


class _Scan(torch.autograd.Function):
    @staticmethod
    def forward(ctx, a, b, init):
        b = b.to(a.dtype)
        a, b, init = a.contiguous(), b.contiguous(), init.contiguous()
        _check(a, b, init)
        batch, steps, features = a.shape
        h = torch.empty_like(a)
        _lib.check(_lib.lib().bt_linear_scan(
            _ptr(a), _ptr(b), _ptr(init), _ptr(h), batch, steps, features, _DTYPES[a.dtype],
            _DTYPES[init.dtype], _stream()))
        ctx.save_for_backward(a, h, init)
        return h

    @staticmethod
    def backward(ctx, cot):
        a, h, init = ctx.saved_tensors
        cot = cot.to(a.dtype).contiguous()
        batch, steps, features = a.shape
        da, db = torch.empty_like(a), torch.empty_like(a)
        dinit = torch.empty_like(init)
        _lib.check(_lib.lib().bt_linear_scan_backward(
            _ptr(a), _ptr(h), _ptr(init), _ptr(cot), _ptr(da), _ptr(db), _ptr(dinit), batch,
            steps, features, _DTYPES[a.dtype], _DTYPES[init.dtype], _stream()))
        return da, db, dinit


def scan(a: torch.Tensor, b: torch.Tensor, init: torch.Tensor) -> torch.Tensor:
    if a.ndim == 3:
        return _Scan.apply(a, b, init)
    batch, steps, *extra, features = a.shape

    def fold(x):
        return torch.movedim(x, 1, -2).reshape(-1, steps, features)

    out = _Scan.apply(fold(a), fold(b), init.reshape(-1, features))
    return torch.movedim(out.reshape(batch, *extra, steps, features), -2, 1)


def sequential(a, b, init):
    """scan.py:119-131 in torch: a float32 carry over the steps, outputs in a's dtype."""
    h = init.float()
    outs = []
    for t in range(a.shape[1]):
        h = a[:, t].float() * h + b[:, t].float()
        outs.append(h.to(a.dtype))
    return torch.stack(outs, 1)


def associative(a, b, init):
    """scan.py:106-116 in its closed form: the prefix maps (cumulative products of a, the scan
    of b from a zero carry) applied to init, in float32 (or wider)."""
    dtype = torch.promote_types(torch.promote_types(a.dtype, b.dtype), torch.float32)
    a, b, init = a.to(dtype), b.to(dtype), init.to(dtype)
    return sequential(a, b, torch.zeros_like(init)) + torch.cumprod(a, 1) * init[:, None]


IMPLEMENTATIONS = {"cuda": scan, "sequential": sequential, "associative": associative}


def get_scan_implementation(name: str | None = None):
    if name is None:
        return scan
    if name not in IMPLEMENTATIONS:
        raise KeyError(f"unknown scan implementation {name!r}, have {sorted(IMPLEMENTATIONS)}")
    return IMPLEMENTATIONS[name]
