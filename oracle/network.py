"""Actor-critic forward and analytic backward (test infrastructure only).

Restates the networks the PPO recipes build with flax (hangar/recipes/ppo_*.py):
`Network` -> `FeatureExtractor` -> `nn.Sequential` of Dense / Conv / LayerNorm /
activation (boonta/networks/network.py:19-49, feature_extractor.py:16-31), and the heads
of boonta/networks/actor_critic.py:7-14 with distributions.py:8-57.

flax semantics restated (flax 0.12.8 is not vendored or installed):
  * Dense: z = x @ kernel + bias, kernel [in, out].
  * Conv(features, (3, 3), padding="SAME"), NHWC, cross-correlation, kernel [3, 3, in, out].
  * LayerNorm (epsilon 1e-6, use_fast_variance=True): mean = E[z], var = max(E[z^2] -
    E[z]^2, 0), y = (z - mean) * (rsqrt(var + eps) * scale) + bias.
  * activations: tanh, relu (gradient 0 at 0, as jax.nn.relu), silu(z) = z * sigmoid(z).

`precision="bf16"` rounds both GEMM operands (the layer input and the kernel in the
forward pass; the output gradient and the kernel/input in the backward pass) to bfloat16
with round-to-nearest-even before an fp32 product, the arithmetic of the CUDA path's bf16
tensor-core GEMMs (whose dW GEMM also yields the bias gradient, as the sum of the
bf16-rounded output gradient). The forward bias add, LayerNorm, activations and the heads
stay fp32. Convolutions always run in fp32.
"""
from __future__ import annotations

import numpy as np

from boonta_b200.spec import Conv3x3, Dense, NetworkSpec

LN_EPS = 1e-6


def bf16_round(x: np.ndarray) -> np.ndarray:
    """Round float32 to the nearest bfloat16 (ties to even), returned as float32."""
    x = np.ascontiguousarray(x, np.float32)
    u = x.view(np.uint32).astype(np.uint64)
    u = (u + 0x7FFF + ((u >> 16) & 1)) & 0xFFFF0000
    return u.astype(np.uint32).view(np.float32).reshape(x.shape)


def quantize(x, precision):
    """bf16 operands: x rounded to float32 and then to bfloat16, returned in x's own dtype (so
    that a float64 evaluation multiplies the bf16 values exactly)."""
    if precision == "bf16":
        x = np.asarray(x)
        return bf16_round(x.astype(np.float32)).astype(x.dtype, copy=False)
    return x


def activation(z, kind):
    if kind == "none":
        return z
    if kind == "tanh":
        return np.tanh(z)
    if kind == "relu":
        return np.maximum(z, 0).astype(z.dtype)
    if kind == "silu":
        return z * sigmoid(z)
    raise ValueError(kind)


def sigmoid(z):
    one = z.dtype.type(1)
    return one / (one + np.exp(-z))


def activation_grad(z, h, kind):
    """d activation / d z, evaluated from the pre-activation z and output h."""
    one = z.dtype.type(1)
    if kind == "none":
        return np.ones_like(z)
    if kind == "tanh":
        return one - h * h
    if kind == "relu":
        return (z > 0).astype(z.dtype)
    if kind == "silu":
        s = sigmoid(z)
        return s * (one + z * (one - s))
    raise ValueError(kind)


def layernorm_forward(z, scale, bias, eps=LN_EPS):
    dt = z.dtype.type
    mean = z.mean(-1, keepdims=True)
    mean2 = (z * z).mean(-1, keepdims=True)
    var = np.maximum(mean2 - mean * mean, dt(0))
    r = dt(1) / np.sqrt(var + dt(eps))
    xhat = (z - mean) * r
    y = (z - mean) * (r * scale) + bias
    return y, (xhat, r)


def layernorm_backward(dy, scale, cache):
    xhat, r = cache
    dscale = (dy * xhat).sum(0)
    dbias = dy.sum(0)
    dxhat = dy * scale
    n = dy.shape[-1]
    m1 = dxhat.sum(-1, keepdims=True) / n
    m2 = (dxhat * xhat).sum(-1, keepdims=True) / n
    dz = r * (dxhat - m1 - xhat * m2)
    return dz, dscale, dbias


def im2col3x3(img):
    """img [M, H, W, C] -> columns [M, H, W, 9*C] in (dy, dx, c) order, SAME padding."""
    m, h, w, c = img.shape
    pad = np.zeros((m, h + 2, w + 2, c), img.dtype)
    pad[:, 1:-1, 1:-1] = img
    cols = np.empty((m, h, w, 9, c), img.dtype)
    for dy in range(3):
        for dx in range(3):
            cols[:, :, :, dy * 3 + dx] = pad[:, dy : dy + h, dx : dx + w]
    return cols.reshape(m, h, w, 9 * c)


def forward(spec: NetworkSpec, params: dict, obs: np.ndarray, precision: str = "fp32"):
    """Returns (actor_out [M, A], value [M], cache). actor_out is the logits
    (categorical) or the gaussian mean."""
    dtype = obs.dtype
    towers = spec.towers()
    names = ["torso"] if spec.shared else ["actor", "critic"]
    cache = {"obs": obs, "towers": []}
    feats = []
    for tname, tower in zip(names, towers):
        h = obs
        layers = []
        for i, layer in enumerate(tower):
            p = f"{tname}/{i}"
            kernel = params[f"{p}/kernel"].astype(dtype)
            bias = params[f"{p}/bias"].astype(dtype)
            ent = {"layer": layer, "prefix": p}
            if isinstance(layer, Conv3x3):
                img = h.reshape(-1, layer.height, layer.width, layer.in_channels)
                cols = im2col3x3(img).reshape(-1, 9 * layer.in_channels)
                x_in = cols
                k2 = kernel.reshape(9 * layer.in_channels, layer.features)
                z = cols @ k2 + bias
                z = z.reshape(h.shape[0], -1)
            elif isinstance(layer, Dense):
                x_in = h
                z = quantize(h, precision) @ quantize(kernel, precision) + bias
            else:
                raise TypeError(layer)
            ent["x"] = x_in
            ent["z"] = z
            pre = z
            if getattr(layer, "layernorm", False):
                y, ln_cache = layernorm_forward(
                    z, params[f"{p}/ln_scale"].astype(dtype), params[f"{p}/ln_bias"].astype(dtype)
                )
                ent["ln"] = ln_cache
                ent["y"] = y
                pre = y
            h = activation(pre, layer.activation)
            ent["pre"] = pre
            ent["h"] = h
            layers.append(ent)
        cache["towers"].append(layers)
        feats.append(h)
    f_pi = feats[0]
    f_v = feats[0] if spec.shared else feats[1]
    cache["f_pi"], cache["f_v"] = f_pi, f_v
    out = f_pi @ params["actor_head/kernel"].astype(dtype) + params["actor_head/bias"].astype(dtype)
    value = (f_v @ params["critic_head/kernel"].astype(dtype) + params["critic_head/bias"].astype(dtype))[:, 0]
    return out, value, cache


def backward(spec: NetworkSpec, params: dict, cache, d_out, d_value, precision: str = "fp32"):
    """Gradients of every parameter given dL/d(actor_out) [M, A] and dL/d(value) [M]."""
    dtype = d_out.dtype
    grads = {}
    f_pi, f_v = cache["f_pi"], cache["f_v"]
    grads["actor_head/kernel"] = f_pi.T @ d_out
    grads["actor_head/bias"] = d_out.sum(0)
    dv = d_value[:, None]
    grads["critic_head/kernel"] = f_v.T @ dv
    grads["critic_head/bias"] = dv.sum(0)
    d_fpi = d_out @ params["actor_head/kernel"].astype(dtype).T
    d_fv = dv @ params["critic_head/kernel"].astype(dtype).T
    names = ["torso"] if spec.shared else ["actor", "critic"]
    d_feats = [d_fpi + d_fv] if spec.shared else [d_fpi, d_fv]
    for tname, tower, layers, dh in zip(names, spec.towers(), cache["towers"], d_feats):
        for i in reversed(range(len(tower))):
            layer = tower[i]
            ent = layers[i]
            p = ent["prefix"]
            dpre = dh * activation_grad(ent["pre"], ent["h"], layer.activation)
            if getattr(layer, "layernorm", False):
                dz, dscale, dbias = layernorm_backward(
                    dpre, params[f"{p}/ln_scale"].astype(dtype), ent["ln"]
                )
                grads[f"{p}/ln_scale"] = dscale
                grads[f"{p}/ln_bias"] = dbias
            else:
                dz = dpre
            kernel = params[f"{p}/kernel"].astype(dtype)
            if isinstance(layer, Conv3x3):
                dzc = dz.reshape(-1, layer.features)
                k2 = kernel.reshape(9 * layer.in_channels, layer.features)
                grads[f"{p}/kernel"] = (ent["x"].T @ dzc).reshape(kernel.shape)
                grads[f"{p}/bias"] = dzc.sum(0)
                if i > 0:
                    raise NotImplementedError("a conv layer is only supported as the first layer")
            else:
                grads[f"{p}/kernel"] = quantize(ent["x"], precision).T @ quantize(dz, precision)
                # the bias gradient rides the dW GEMM as a ones row of the input, so in
                # bf16 mode it sums the bf16-rounded dz
                grads[f"{p}/bias"] = quantize(dz, precision).sum(0)
                if i > 0:
                    dh = quantize(dz, precision) @ quantize(kernel, precision).T
    return grads
