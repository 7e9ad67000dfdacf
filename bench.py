"""Benchmark of the PPO learner step (boonta PPO.update) on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--config c5] [--impl native|reference]

Metric: learner env-steps/s = world * T * N / t_update (the reference's `update/SPS`,
hangar/scripts/benchmark_boonta.py:154-177, 214), weak scaling (N envs per GPU fixed).
One "step" = one full learner update: bootstrap value, GAE, E x M minibatch
forward/loss/backward/(all-reduce)/clip+Adam. Inputs are seeded synthetic rollouts of the
workload's shapes, resident in HBM when the timed region starts (`value`); `e2e` repeats
the measurement through the public API with the rollout copied from pinned host memory
and the statistics read back every step. Every timed rollout and its permutations are
larger than L2 (126 MB), and each step uses a different permutation. The line also carries
`act`: the act step (PPO.step) through Learner.act over one rollout step's N envs, device-timed
(not part of `value`).

`--impl reference` times the reference's algorithm on the host cores. boonta's own JAX
path cannot run here (no jax/flax/optax in the image), so it times the NumPy port of it
(oracle/, the CPU restatement the parity tests check against) on a bounded sample of the
same workload and scales it to one full update.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import time
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

from boonta_b200 import configs  # noqa: E402
from boonta_b200.spec import GRU, Conv3x3, Dense, init_params, param_layout  # noqa: E402

PEAKS_FALLBACK = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}


def peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return d, "measured"
    return PEAKS_FALLBACK, "fallback"


# ---- algorithmic work per update, by kernel class ---------------------------------------
def class_work(w) -> dict:
    """{kernel class: (FLOPs, bytes)} of one learner update, counted algorithmically: every
    GEMM as 2*M*N*K (the split-bf16 mode issues three products per term; they are not
    counted), every operand read once and every output written once, in the precision the
    path stores it (bf16 2 B, split-bf16 pairs 4 B, fp32 4 B). A GRU layer (fp32) counts its
    input projection [x, 1] W_i and its recurrence h W_h (forward), the recurrence's carry
    products and the GRU input's gradient (dX), and the three weight gradients (dW); its
    gate arithmetic is not counted."""
    net = w.network
    # rows of one minibatch: samples, or whole env sequences times T (recurrent)
    rows = w.minibatch_size * (w.num_steps if net.recurrent else 1)
    steps = w.ppo.update_epochs * w.ppo.num_minibatches
    tc = w.precision in ("bf16", "bf16x3")
    e = {"fp32": 4, "bf16": 2, "bf16x3": 4}[w.precision]
    out = {k: [0.0, 0.0] for k in ("gemm_fwd", "gemm_dx", "gemm_dw", "heads_loss", "head_dw")}
    feats = []
    for tower in net.towers():
        dim = net.obs_dim
        for i, layer in enumerate(tower):
            last = i + 1 == len(tower)
            if isinstance(layer, GRU):
                h = layer.features
                g3 = 3 * h
                out["gemm_fwd"][0] += 2.0 * rows * ((dim + 1) * g3 + h * g3)
                # x read, xp written and re-read, the carry-in, output and three gates written
                out["gemm_fwd"][1] += rows * (dim * 4 + g3 * 8 + 5 * h * 4) + ((dim + 1) + h) * g3 * 4
                out["gemm_dx"][0] += 2.0 * rows * (h * g3 + dim * g3)
                out["gemm_dx"][1] += rows * (g3 * 8 + 6 * h * 4 + dim * 4) + (h + dim) * g3 * 4
                out["gemm_dw"][0] += 2.0 * rows * ((dim + 1) * g3 + h * g3 + h)
                out["gemm_dw"][1] += rows * (dim * 4 + g3 * 8 + 2 * h * 4) + ((dim + 1) + h + 1) * g3 * 4
                dim = h
                continue
            if isinstance(layer, Conv3x3):
                m = rows * layer.height * layer.width
                k, n = 9 * layer.in_channels + 1, layer.features
                width = layer.height * layer.width * layer.features
                a_bytes = rows * dim * 4
            else:
                m, k, n = rows, dim + 1, layer.features
                width = n
                a_bytes = rows * dim * (e if tc else 4)
            w_bytes = k * n * (e if tc else 4)
            # z (fp32) and the layer output: bf16 (pair) for the next tensor-core layer, none
            # after a tensor-core tower's last layer (the heads read z), fp32 otherwise
            out_fwd = rows * width * (4 + ((0 if last else e) if tc else 4))
            out["gemm_fwd"][0] += 2.0 * m * k * n
            out["gemm_fwd"][1] += a_bytes + w_bytes + out_fwd
            dz_bytes = rows * width * (e if tc else 4)
            out["gemm_dw"][0] += 2.0 * m * k * n
            out["gemm_dw"][1] += dz_bytes + a_bytes + k * n * 4
            if i > 0:
                out["gemm_dx"][0] += 2.0 * m * (k - 1) * n
                out["gemm_dx"][1] += dz_bytes + w_bytes + rows * dim * (4 + (e if tc else 4))
            dim = width
        feats.append(dim)
    f_pi = feats[0]
    f_v = feats[-1]
    a = net.action_dim
    nf = f_pi + (0 if net.shared else f_v)
    # heads: features + pre-activations read, dz written, head outputs' gradients written
    out["heads_loss"][0] += 2.0 * rows * (f_pi * a + f_v) * 2
    out["heads_loss"][1] += rows * nf * (4 + 4 + (e if tc else 4)) + rows * (a + 1) * 4 + rows * 20
    # head weight gradients: [f, 1]^T d_out and [f, 1]^T d_value (features re-read)
    out["head_dw"][0] += 2.0 * rows * ((f_pi + 1) * a + (f_v + 1))
    out["head_dw"][1] += rows * (f_pi + f_v) * 4 + rows * (a + 1) * 4
    return {k: (v[0] * steps, v[1] * steps) for k, v in out.items()}


def class_table(w, prof: dict, pk: dict) -> dict:
    """Every profiled kernel class with its device time per update, achieved TFLOP/s against
    the measured sustained bf16 peak and achieved GB/s of algorithmic bytes against the
    measured copy bandwidth."""
    work = class_work(w)
    tflops_peak = pk.get("bf16_tflops_sustained", pk.get("bf16_tflops"))
    out = {}
    for cls, (ms, n) in sorted(prof.items(), key=lambda kv: -kv[1][0]):
        row = {"ms": ms, "launches": n}
        if cls in work and ms > 0:
            flops, nbytes = work[cls]
            row["tflops"] = flops / (ms / 1e3) / 1e12
            row["frac_bf16_sustained"] = row["tflops"] / tflops_peak
            row["gbs"] = nbytes / (ms / 1e3) / 1e9
            row["frac_hbm"] = row["gbs"] / pk["hbm_gbs"]
        out[cls] = row
    return out


def roofline(w, prof: dict, pk: dict, pk_kind: str) -> dict:
    """Roofline of the class with the most device time: its algorithmic FLOPs and bytes per
    update against the measured bf16 tensor peak and HBM copy bandwidth; the bound is the
    resource whose roofline time is longer."""
    work = class_work(w)
    if not prof:
        return {"bound": None, "achieved": None, "peak": None, "unit": None, "frac": None,
                "traffic": None}
    cls, (ms, n) = max(prof.items(), key=lambda kv: kv[1][0])
    sec = ms / 1000.0
    tflops_peak = pk.get("bf16_tflops_sustained", pk.get("bf16_tflops"))
    gbs_peak = pk["hbm_gbs"]
    line = {"kernel": cls, "launches": n, "device_ms": ms, "peaks": pk_kind}
    if cls in work:
        flops, nbytes = work[cls]
        t_tensor = flops / (tflops_peak * 1e12)
        t_hbm = nbytes / (gbs_peak * 1e9)
        if t_tensor >= t_hbm:
            ach = flops / sec / 1e12
            line.update(bound="tensor", achieved=ach, peak=tflops_peak, unit="TFLOP/s",
                        frac=ach / tflops_peak, algorithmic_per_launch=flops / n)
        else:
            ach = nbytes / sec / 1e9
            line.update(bound="hbm", achieved=ach, peak=gbs_peak, unit="GB/s",
                        frac=ach / gbs_peak, algorithmic_per_launch=nbytes / n)
    else:
        line.update(bound="hbm", achieved=None, peak=gbs_peak, unit="GB/s", frac=None)
    cap = TRAFFIC.get((w.name, w.precision, cls))
    line["traffic"] = None
    if cap and "algorithmic_per_launch" in line:
        # the captured launch's DRAM bytes, scaled to the class's average launch by the ratio
        # of algorithmic bytes (traffic grows in proportion to the rows and widths processed)
        line["traffic"] = cap[0] * (nbytes / n) / cap[1]
    return line


# {(workload, precision, class): (dram__bytes_read.sum + dram__bytes_write.sum of one captured
# launch, that launch's algorithmic bytes)}, from the ncu --set full captures summarised in
# profiles/<class>_<workload>_<precision>.md.
TRAFFIC = {
    ("c2_brax", "bf16x3", "gemm_fwd"): (17.93e6, 50.6e6),   # a 256-wide layer; outputs stay in L2
    ("c2_brax", "bf16x3", "gemm_dx"): (33.96e6, 50.6e6),    # a 256-wide layer; outputs stay in L2
    ("c2_brax", "bf16x3", "gemm_dw"): (34.11e6, 39.9e6),    # a 256-wide layer
    ("c2_brax", "bf16x3", "heads_loss"): (43.23e6, 101.6e6),
}


def gae_bytes(w) -> float:
    return 18.0 * w.batch_size + 4.0 * w.num_envs


def gae_bandwidth(w, device, rounds: int = 4) -> dict:
    """HBM bandwidth of the GAE kernel alone on the workload's [T, N] shape, through the public
    bt_gae entry point: back-to-back launches cycling over enough independent copies of the
    inputs and outputs that their total (> 160 MB) exceeds L2, so every launch reads and writes
    HBM; CUDA events around `rounds` passes over the copies, after one untimed pass."""
    import ctypes

    import torch

    from boonta_b200 import _lib

    lib = _lib.lib()
    t, n = w.num_steps, w.num_envs
    per = gae_bytes(w)
    copies = min(64, max(2, int(np.ceil(160e6 / per))))
    g = torch.Generator(device=device)
    g.manual_seed(5)
    bufs = []
    for _ in range(copies):
        bufs.append((torch.randn((t, n), generator=g, device=device),
                     (torch.rand((t, n), generator=g, device=device) < w.done_p).to(torch.uint8),
                     torch.zeros((t, n), dtype=torch.uint8, device=device),
                     torch.randn((t, n), generator=g, device=device),
                     torch.randn((n,), generator=g, device=device),
                     torch.empty((t, n), device=device), torch.empty((t, n), device=device)))
    stream = torch.cuda.current_stream()
    sp = ctypes.c_void_p(stream.cuda_stream)

    def one(b):
        _lib.check(lib.bt_gae(*(x.data_ptr() for x in b[:5]), None, None, t, n,
                              float(w.ppo.gamma), float(w.ppo.gae_lambda), b[5].data_ptr(),
                              b[6].data_ptr(), sp))

    for b in bufs:
        one(b)
    torch.cuda.synchronize()
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record(stream)
    for _ in range(rounds):
        for b in bufs:
            one(b)
    e.record(stream)
    torch.cuda.synchronize()
    us = s.elapsed_time(e) * 1000.0 / (rounds * copies)
    gbs = per / (us * 1e-6) / 1e9
    pk, pk_kind = peaks()
    del bufs
    return {"gbs": gbs, "us_per_launch": us, "bytes_per_launch": per, "launches": rounds * copies,
            "frac": gbs / pk["hbm_gbs"], "peak": pk["hbm_gbs"], "peaks": pk_kind,
            "note": f"{copies} input/output copies cycled (> L2), back-to-back launches"}


# ---- synthetic inputs on the device ----------------------------------------------------------
def act_timing(w, lrn, roll, device, calls: int = 32) -> dict:
    """The act step (PPO.step, ppo.py:57-74) through the public Learner.act /
    Learner.act_recurrent over the N envs of one rollout step, as the rollout loop of
    anakin.py:46-76 calls it: device time per call (CUDA events around `calls` back-to-back
    calls, after 3 untimed ones) cycling over the rollout's T observation slices, with uniform
    (categorical) or normal (gaussian) noise drawn on the device beforehand."""
    import torch

    t, n, a = w.num_steps, w.num_envs, w.network.action_dim
    g = torch.Generator(device=device)
    g.manual_seed(11)
    noise = (torch.rand((calls, n, a), generator=g, device=device).clamp_(min=1e-30)
             if w.network.head == "categorical"
             else torch.randn((calls, n, a), generator=g, device=device))
    obs = roll["obs"]
    if w.network.recurrent:
        h = w.network.towers()[0][-1].features
        carry = torch.zeros((n, h), device=device)
        reset = torch.zeros(n, dtype=torch.uint8, device=device)
        call = lambda i: lrn.act_recurrent(obs[i % t], reset, carry, noise[i])
    else:
        call = lambda i: lrn.act(obs[i % t], noise[i])
    for i in range(3):
        call(i)
    torch.cuda.synchronize()
    l0 = lrn.launch_count()
    stream = torch.cuda.current_stream()
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record(stream)
    for i in range(calls):
        call(i)
    e.record(stream)
    torch.cuda.synchronize()
    ms = s.elapsed_time(e) / calls
    return {"ms_per_call": ms, "env_steps_per_s": n / (ms / 1000.0), "rows": n,
            "gpu_launches_per_call": (lrn.launch_count() - l0) / calls,
            "note": "device time of Learner.act over one rollout step's N envs (network "
                    "forward, heads, sampling fused into the heads kernel)"}


def device_rollout(w, seed: int, device):
    import torch

    g = torch.Generator(device=device)
    g.manual_seed(seed)
    t, n, d, a = w.num_steps, w.num_envs, w.network.obs_dim, w.network.action_dim

    def obs(shape):
        if w.obs_kind == "bernoulli":
            return (torch.rand(shape, generator=g, device=device) < 1 - w.obs_sparsity).float()
        if w.obs_kind == "sparse_uniform":
            x = torch.rand(shape, generator=g, device=device)
            keep = torch.rand(shape, generator=g, device=device) >= w.obs_sparsity
            return torch.where(keep, x, torch.zeros((), device=device))
        return torch.randn(shape, generator=g, device=device)

    r = {"obs": obs((t, n, d)), "bootstrap_obs": obs((n, d))}
    if w.network.head == "gaussian":
        r["action"] = torch.randn((t, n, a), generator=g, device=device)
        r["log_prob"] = (-0.5 * r["action"] ** 2 - 0.9189385).sum(-1) + 0.05 * torch.randn(
            (t, n), generator=g, device=device)
    else:
        r["action"] = torch.randint(0, a, (t, n), generator=g, device=device, dtype=torch.int32)
        r["log_prob"] = float(np.log(1.0 / a)) + 0.05 * torch.randn((t, n), generator=g, device=device)
    if w.reward == "ones":
        r["reward"] = torch.ones((t, n), device=device)
    elif w.reward == "bernoulli":
        r["reward"] = (torch.rand((t, n), generator=g, device=device) < w.reward_p).float()
    else:
        r["reward"] = w.reward_scale * torch.randn((t, n), generator=g, device=device)
    r["terminated"] = (torch.rand((t, n), generator=g, device=device) < w.done_p).to(torch.uint8)
    r["truncated"] = torch.zeros((t, n), dtype=torch.uint8, device=device)
    r["value"] = torch.randn((t, n), generator=g, device=device)
    if w.network.recurrent:
        # first.done (reset before step t), the carry entering step 0 and step T-1
        h = w.network.torso[-1].features
        fd = torch.zeros((t, n), dtype=torch.uint8, device=device)
        fd[0] = (torch.rand(n, generator=g, device=device) < w.done_p).to(torch.uint8)
        fd[1:] = r["terminated"][:-1] | r["truncated"][:-1]
        r["first_done"] = fd
        r["carry"] = w.hidden_std * torch.randn((n, h), generator=g, device=device)
        r["last_carry"] = w.hidden_std * torch.randn((n, h), generator=g, device=device)
    return {k: v.contiguous() for k, v in r.items()}


def device_perms(w, world: int, count: int, seed: int, device):
    import torch

    g = torch.Generator(device=device)
    g.manual_seed(seed)
    # recurrent networks permute environments (env-minibatches), the others samples
    size = (w.num_envs if w.network.recurrent else w.batch_size) * world
    return [torch.stack([torch.randperm(size, generator=g, device=device, dtype=torch.int32)
                         for _ in range(w.ppo.update_epochs)]) for _ in range(count)]


# ---- clocks ---------------------------------------------------------------------------------
class ClockSampler:
    QUERY = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.gpu}", f"--query-gpu={self.QUERY}",
                 "--format=csv,noheader,nounits", "-lms", "100"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except Exception:
            self.proc = None
        return self

    def __exit__(self, *exc):
        self.lines = []
        if self.proc is not None:
            time.sleep(0.25)
            self.proc.terminate()
            try:
                out, _ = self.proc.communicate(timeout=5)
            except Exception:
                self.proc.kill()
                out = ""
            self.lines = [line for line in out.splitlines() if line.strip()]

    def summary(self) -> dict:
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in getattr(self, "lines", []):
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                mx = float(parts[2])
            except ValueError:
                continue
            for name, val in zip(names, parts[5:9]):
                if val.lower() == "active":
                    reasons.add(name)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx,
                "reasons": sorted(reasons), "samples": len(sm)}


# ---- CPU baseline (the reference's algorithm on the host) -----------------------------------
def host_threads() -> int:
    return len(os.sched_getaffinity(0))


def bench_config(w, world: int) -> dict:
    """The workload description both arms print (identical keys and values)."""
    return {"workload": w.name, "T": w.num_steps, "N_per_gpu": w.num_envs,
            "epochs": w.ppo.update_epochs, "minibatches": w.ppo.num_minibatches,
            "minibatch_rows": w.minibatch_size * (w.num_steps if w.network.recurrent else 1),
            "precision": w.precision, "parallelism": f"dp{world}",
            "l2": ("inputs larger than L2 (obs rollout "
                   f"{w.batch_size * w.network.obs_dim * 4 / 1e6:.0f} MB per GPU)"),
            "description": w.description}


def _host_minibatch(w, seed: int = 77) -> dict:
    """One full-size minibatch of the workload on the host (its rows only), in the oracle's
    input layout: flat samples, or whole env sequences [envs, T] for a recurrent network."""
    if w.network.recurrent:
        sub = w.scaled(num_envs=w.minibatch_size)
        roll = configs.rollout(sub, seed=seed)
        tr = lambda a: np.moveaxis(a, 0, 1)  # [T, N, ...] -> [N, T, ...]
        rng = np.random.default_rng(seed + 1)
        return {"obs": tr(roll["obs"]), "done": tr(roll["first_done"]),
                "action": tr(roll["action"]), "log_prob": tr(roll["log_prob"]),
                "value": tr(roll["value"]),
                "advantages": rng.standard_normal(roll["value"].shape, dtype=np.float32).T,
                "returns": rng.standard_normal(roll["value"].shape, dtype=np.float32).T,
                "carry": roll["carry"]}
    rows = w.minibatch_size
    rng = np.random.default_rng(seed)
    a = w.network.action_dim
    mb = {"obs": configs._obs(rng, w, (rows, w.network.obs_dim))}
    if w.network.head == "gaussian":
        mb["action"] = rng.standard_normal((rows, a), dtype=np.float32)
        mb["log_prob"] = (-0.5 * mb["action"] ** 2 - 0.9189385).sum(-1).astype(np.float32)
    else:
        mb["action"] = rng.integers(0, a, rows, dtype=np.int32)
        mb["log_prob"] = np.full(rows, np.log(1.0 / a), np.float32)
    for k in ("value", "advantages", "returns"):
        mb[k] = rng.standard_normal(rows, dtype=np.float32)
    return mb


_HOST_INPUTS: dict = {}


def _host_inputs(w):
    """The host rollout (without its [T, N, D] observations unless the network is recurrent)
    and one full-size minibatch, made once per workload and reused by every timed sample."""
    if w.name not in _HOST_INPUTS:
        _HOST_INPUTS[w.name] = (configs.rollout(w, include_obs=w.network.recurrent),
                                _host_minibatch(w))
    return _HOST_INPUTS[w.name]


def cpu_baseline(w, budget_s: float = 4.0) -> dict:
    """The reference's algorithm (the NumPy port in oracle/, float32) on the host cores, on a
    bounded sample of one update of the workload: the bootstrap value and GAE over the whole
    [T, N] rollout, then minibatch steps of the full minibatch size (forward, loss, backward,
    clip + Adam) until `budget_s` is spent (at least one). One update's time is extrapolated
    as targets + (E x M) x the mean minibatch step; `value` = T*N / that time."""
    from oracle import gae as ogae
    from oracle import network as onet
    from oracle import optim
    from oracle import ppo as oppo
    from oracle import recurrent as orec

    threads = host_threads()
    try:
        from threadpoolctl import threadpool_limits

        limiter = threadpool_limits(limits=threads)
    except Exception:
        limiter = None
    params = init_params(w.network, seed=0, init=w.init)
    opt_state = optim.init_state(params)
    roll, mb = _host_inputs(w)
    wall0 = time.perf_counter()
    t0 = time.perf_counter()
    if w.network.recurrent:
        seq_obs = np.stack([roll["obs"][-1], roll["bootstrap_obs"]], axis=1)
        second_done = roll["terminated"][-1] | roll["truncated"][-1]
        seq_done = np.stack([roll["first_done"][-1], second_done], axis=1)
        _, v2, _ = orec.forward_seq(w.network, params, seq_obs, seq_done, roll["last_carry"])
        boot = v2[:, -1]
    else:
        _, boot, _ = onet.forward(w.network, params, roll["bootstrap_obs"])
    ogae.gae(roll["reward"], roll["terminated"], roll["truncated"], roll["value"], boot,
             w.ppo.gamma, w.ppo.gae_lambda)
    t_targets = time.perf_counter() - t0
    done, t_mb = 0, 0.0
    total = w.ppo.update_epochs * w.ppo.num_minibatches
    while done < total:
        t0 = time.perf_counter()
        if w.network.recurrent:
            traj = {k: v for k, v in mb.items() if k != "carry"}
            _, _, grads = orec.loss_and_grads(w.network, w.ppo, params, traj, mb["carry"])
        else:
            _, _, grads = oppo.loss_and_grads(w.network, w.ppo, params, mb)
        params, opt_state = optim.clip_adam(params, grads, opt_state, w.optimizer)
        t_mb += time.perf_counter() - t0
        done += 1
        if t_targets + t_mb >= budget_s:
            break
    sample_s = time.perf_counter() - wall0
    if limiter is not None:
        limiter.unregister()
    t_update = t_targets + t_mb / done * total
    return {"value": w.batch_size / t_update, "unit": "env-steps/s", "cores": threads,
            "kind": "port", "sample_s": sample_s, "minibatch_steps_timed": done,
            "minibatch_steps_per_update": total, "extrapolated": done < total,
            "sample": (f"NumPy oracle (float32, {threads} BLAS threads) on the {w.name} workload: "
                       f"bootstrap + GAE over the full T={w.num_steps} x N={w.num_envs} rollout, "
                       f"then {done} of the update's {total} minibatch steps at the full "
                       f"minibatch size; one update's time extrapolated as targets + "
                       f"{total} x the mean minibatch step")}


def run_reference(args, w):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    steps, samples = [], []
    cb = None
    for _ in range(args.warmup + args.steps):
        cb = cpu_baseline(w)
        steps.append(cb["value"])
        samples.append(cb["sample_s"])
    timed = steps[args.warmup:] or steps[-1:]
    value = statistics.median(timed)
    cb["value"] = value
    sample_ms = 1000.0 * statistics.mean(samples[args.warmup:] or samples[-1:])
    line = {
        "impl": "reference", "metric": "ppo_learner_env_steps_per_sec", "value": value,
        "unit": "env-steps/s", "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        # each step is the bounded sample above, timed on the host; one full update's time
        # is extrapolated from it (extrapolated_update_ms)
        "ms_per_step": sample_ms, "extrapolated_update_ms": 1000.0 * w.batch_size / value,
        "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": bench_config(w, args.gpus),
        "cpu_baseline": cb,
        "e2e": {"value": value, "unit": "env-steps/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--config", default="c5")
    ap.add_argument("--precision", default=None)
    ap.add_argument("--impl", default="native", choices=["native", "reference"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-p2p", action="store_true",
                    help="multi-GPU: NCCL all-reduce + full optimizer step instead of the NVLink "
                         "peer-memory exchange")
    ap.add_argument("--no-profile", action="store_true",
                    help="skip the per-kernel-class profiled pass (for ncu launch lists)")
    ap.add_argument("--num-envs", type=int, default=None,
                    help="fewer environments per GPU (a small case for profiler captures; with "
                         "--minibatches, the same minibatch shape on a smaller rollout)")
    ap.add_argument("--minibatches", type=int, default=None)
    args = ap.parse_args()

    kw = {"precision": args.precision} if args.precision else {}
    w = configs.make(args.config, **kw)
    scale = {k: v for k, v in (("num_envs", args.num_envs),
                               ("num_minibatches", args.minibatches)) if v}
    if scale:
        w = w.scaled(**scale)
    if args.impl == "reference":
        return run_reference(args, w)

    import torch
    import torch.distributed as dist

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    device = torch.device("cuda", local)
    if world > 1:
        from datetime import timedelta

        dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=device)

    from boonta_b200.learner import Learner

    lrn = Learner.from_workload(w, world_size=world, rank=rank)
    if world > 1:
        uid = torch.zeros(128, dtype=torch.uint8, device=device)
        if rank == 0:
            uid.copy_(torch.frombuffer(bytearray(Learner.nccl_unique_id()), dtype=torch.uint8))
        dist.broadcast(uid, 0)
        lrn.comm_init(bytes(uid.cpu().numpy()))
        if args.no_p2p:
            lrn.use_p2p(False)
    lrn.set_state(init_params(w.network, seed=0, init=w.init))

    roll = device_rollout(w, seed=100 + rank, device=device)
    n_perm = args.warmup + args.steps
    perms = device_perms(w, world, n_perm, seed=7, device=device)
    stream = torch.cuda.current_stream()

    def barrier():
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()

    for i in range(args.warmup):
        lrn.update(roll, perms[i], stats=True)
    barrier()
    launches0 = lrn.launch_count()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clocks:
        start.record(stream)
        for i in range(args.steps):
            lrn.update(roll, perms[args.warmup + i], stats=True)
        end.record(stream)
        torch.cuda.synchronize()
    barrier()
    ms = start.elapsed_time(end) / max(args.steps, 1)
    launches = (lrn.launch_count() - launches0) // max(args.steps, 1)
    t = torch.tensor([ms], device=device)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms = float(t.item())
    value = world * w.batch_size / (ms / 1000.0)

    # Per-kernel-class device time: the same K steps again, with CUDA events recorded around
    # every launch on the stream it is launched on (a second timed region, so the events'
    # host cost cannot touch the headline number).
    prof = {}
    if not args.no_profile:
        lrn.profile(True)
        for i in range(args.steps):
            lrn.update(roll, perms[args.warmup + i], stats=True)
        torch.cuda.synchronize()
        prof = {k: (ms_ / max(args.steps, 1), n_ // max(args.steps, 1))
                for k, (ms_, n_) in lrn.profile_read().items()}
        lrn.profile(False)

    # end to end: rollout from pinned host memory, statistics back to the host, every step
    e2e = None
    if not args.no_e2e:
        host = {k: v.cpu().pin_memory() for k, v in roll.items()}
        dev = {k: torch.empty_like(v) for k, v in roll.items()}
        h2d = sum(v.numel() * v.element_size() for v in host.values())
        st_host = torch.empty((w.ppo.update_epochs, w.ppo.num_minibatches, 8)).pin_memory()
        barrier()
        s2, e2 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s2.record(stream)
        for i in range(args.steps):
            for k in host:
                dev[k].copy_(host[k], non_blocking=True)
            st = lrn.update(dev, perms[args.warmup + i], stats=True)
            st_host.copy_(st, non_blocking=True)
        e2.record(stream)
        torch.cuda.synchronize()
        barrier()
        ms2 = s2.elapsed_time(e2) / max(args.steps, 1)
        t2 = torch.tensor([ms2], device=device)
        if world > 1:
            dist.all_reduce(t2, op=dist.ReduceOp.MAX)
        ms2 = float(t2.item())
        e2e = {"value": world * w.batch_size / (ms2 / 1000.0), "unit": "env-steps/s",
               "h2d_bytes_per_step": int(h2d), "d2h_bytes_per_step": int(st_host.numel() * 4)}

    if rank != 0:
        if world > 1:
            dist.destroy_process_group()
        return

    pk, pk_kind = peaks()
    roof = roofline(w, prof, pk, pk_kind)
    # GAE inside the update (one event-bracketed launch per update, so launch latency is
    # included) and alone, back to back on inputs larger than L2 (the bandwidth figure)
    gae_in_update = None
    if "gae" in prof:
        g_ms, g_n = prof["gae"]
        gae_in_update = gae_bytes(w) / (g_ms / 1000.0 / g_n) / 1e9
    gae_bw = gae_bandwidth(w, device)
    gae_bw["in_update_gbs"] = gae_in_update

    line = {
        "metric": "ppo_learner_env_steps_per_sec", "value": value, "unit": "env-steps/s",
        "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": {"fp32": "f32", "bf16": "bf16", "bf16x3": "bf16x3"}[w.precision],
        "data": "synthetic",
        "config": bench_config(w, world),
        "roofline": roof,
        "classes": class_table(w, prof, pk),
        "gae_hbm_gbs": gae_bw["gbs"],
        "gae": gae_bw,
        "kernel_ms_per_step": {k: v[0] for k, v in sorted(prof.items())},
        "gpu_launches": int(launches),
        "clocks": clocks.summary(),
        "e2e": e2e,
        "act": act_timing(w, lrn, roll, device),
    }
    if world == 1 and not args.no_cpu_baseline:
        line["cpu_baseline"] = cpu_baseline(w)
    print(json.dumps(line), flush=True)
    if world > 1:
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
