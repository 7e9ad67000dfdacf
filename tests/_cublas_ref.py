"""The loss gradient of one minibatch computed the way a framework's generic path computes it on
this GPU (test infrastructure; imported by the GPU parity tests, never by the product).

The network's GEMMs take bf16 operands and accumulate in fp32 through cuBLAS
(torch.mm(..., out_dtype=float32)), which is what an XLA program of the reference's bf16
networks runs on a B200; everything else (LayerNorm, activations, heads, the PPO loss of
boonta/algorithms/ppo.py:77-146) is fp32 torch with TF32 off, and the gradient comes from
autograd. Its distance from the float64 oracle measures how far bf16 tensor-core arithmetic
with fp32 accumulation lands from exact bf16 arithmetic on this hardware: the noise floor the
bf16 parity bounds are set against (tests/_parity.py).

Only Dense (+ LayerNorm) towers are covered (the bf16 workloads' networks).
"""
import math

import numpy as np


class _Bf16Linear:
    @staticmethod
    def make():
        import torch

        class F(torch.autograd.Function):
            @staticmethod
            def forward(ctx, x, w, b):
                xb, wb = x.to(torch.bfloat16), w.to(torch.bfloat16)
                ctx.save_for_backward(xb, wb)
                return torch.mm(xb, wb, out_dtype=torch.float32) + b

            @staticmethod
            def backward(ctx, dz):
                xb, wb = ctx.saved_tensors
                dzb = dz.to(torch.bfloat16)
                dx = torch.mm(dzb, wb.t(), out_dtype=torch.float32)
                dw = torch.mm(xb.t(), dzb, out_dtype=torch.float32)
                return dx, dw, dzb.float().sum(0)

        return F


def _act(z, kind):
    import torch

    if kind == "tanh":
        return torch.tanh(z)
    if kind == "relu":
        return torch.relu(z)
    if kind == "silu":
        return z * torch.sigmoid(z)
    return z


def supported(spec) -> bool:
    from boonta_b200.spec import Dense

    return all(isinstance(layer, Dense) for tower in spec.towers() for layer in tower)


def loss_and_grads(spec, ppo, params, mb):
    """(stats [8], {name: gradient}) of one minibatch, as numpy arrays."""
    import torch

    from boonta_b200.spec import Dense

    torch.backends.cuda.matmul.allow_tf32 = False
    lin = _Bf16Linear.make()
    dev = torch.device("cuda")
    p = {k: torch.tensor(np.asarray(v, np.float32), device=dev, requires_grad=True)
         for k, v in params.items()}
    obs = torch.tensor(np.asarray(mb["obs"], np.float32), device=dev)
    names = ["torso"] if spec.shared else ["actor", "critic"]
    feats = []
    for tname, tower in zip(names, spec.towers()):
        h = obs
        for i, layer in enumerate(tower):
            assert isinstance(layer, Dense), "dense towers only"
            pre = f"{tname}/{i}"
            z = lin.apply(h, p[f"{pre}/kernel"], p[f"{pre}/bias"])
            if layer.layernorm:
                mean = z.mean(-1, keepdim=True)
                var = torch.clamp((z * z).mean(-1, keepdim=True) - mean * mean, min=0.0)
                z = (z - mean) * (torch.rsqrt(var + 1e-6) * p[f"{pre}/ln_scale"]) + p[f"{pre}/ln_bias"]
            h = _act(z, layer.activation)
        feats.append(h)
    f_pi, f_v = feats[0], feats[-1]
    out = f_pi @ p["actor_head/kernel"] + p["actor_head/bias"]
    value = (f_v @ p["critic_head/kernel"] + p["critic_head/bias"])[:, 0]
    if spec.head == "categorical":
        action = torch.tensor(np.asarray(mb["action"], np.int64), device=dev)
        logp = torch.log_softmax(out, -1)
        lp = logp.gather(1, action[:, None])[:, 0]
        ent = -(logp.exp() * logp).sum(-1)
    else:
        action = torch.tensor(np.asarray(mb["action"], np.float32), device=dev)
        sigma = torch.nn.functional.softplus(p["actor_head/scale"]) + 1e-3
        zz = (action - out) / sigma
        lp = (-0.5 * zz * zz - torch.log(sigma) - 0.5 * math.log(2 * math.pi)).sum(-1)
        ent = (0.5 + 0.5 * math.log(2 * math.pi) + torch.log(sigma)).sum().expand(out.shape[0])
    t = lambda k: torch.tensor(np.asarray(mb[k], np.float32), device=dev)
    lp_old, adv, ret, v_old = t("log_prob"), t("advantages"), t("returns"), t("value")
    eps = ppo.clip_coefficient
    ratio = torch.exp(lp - lp_old)
    actor = -torch.minimum(ratio * adv, torch.clamp(ratio, 1 - eps, 1 + eps) * adv).mean()
    c1 = 0.5 * (value - ret) ** 2
    if ppo.clip_value_loss:
        vc = v_old + torch.clamp(value - v_old, -eps, eps)
        crit = torch.maximum(c1, 0.5 * (vc - ret) ** 2)
    else:
        crit = c1
    critic = crit.mean()
    entropy = ent.mean()
    loss = actor - ppo.entropy_coefficient * entropy + ppo.value_coefficient * critic
    loss.backward()
    with torch.no_grad():
        resid = ret - value
        ev = 1 - resid.var(unbiased=False) / (ret.var(unbiased=False) + 1e-8)
        clipfrac = ((ratio - 1).abs() > eps).float().mean()
        stats = np.array([float(x) for x in (actor, entropy, (lp_old - lp).mean(), clipfrac,
                                              adv.mean(), critic, ev, value.mean())])
    grads = {k: v.grad.double().cpu().numpy() if v.grad is not None else np.zeros(v.shape)
             for k, v in p.items()}
    return stats, grads
