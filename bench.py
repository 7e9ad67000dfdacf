"""Benchmark of the PPO learner step (boonta PPO.update) on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--config c2] [--impl native|reference]

Metric: learner env-steps/s = world * T * N / t_update (the reference's `update/SPS`,
hangar/scripts/benchmark_boonta.py:154-177, 214), weak scaling (N envs per GPU fixed).
One "step" = one full learner update: bootstrap value, GAE, E x M minibatch
forward/loss/backward/(all-reduce)/clip+Adam. Inputs are seeded synthetic rollouts of the
workload's shapes, resident in HBM when the timed region starts (`value`); `e2e` repeats
the measurement through the public API with the rollout copied from pinned host memory
and the statistics read back every step. Every timed rollout and its permutations are
larger than L2 (126 MB), and each step uses a different permutation.

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
from boonta_b200.spec import Conv3x3, Dense, init_params, param_layout  # noqa: E402

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
    path stores it (bf16 2 B, split-bf16 pairs 4 B, fp32 4 B)."""
    net = w.network
    rows = w.minibatch_size
    steps = w.ppo.update_epochs * w.ppo.num_minibatches
    tc = w.precision in ("bf16", "bf16x3")
    e = {"fp32": 4, "bf16": 2, "bf16x3": 4}[w.precision]
    out = {k: [0.0, 0.0] for k in ("gemm_fwd", "gemm_dx", "gemm_dw", "heads_loss", "head_dw")}
    feats = []
    for tower in net.towers():
        dim = net.obs_dim
        for i, layer in enumerate(tower):
            last = i + 1 == len(tower)
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
            out["gemm_dw"][1] += dz_bytes + a_bytes + rows * 0 + k * n * 4
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
def cpu_baseline(w, budget_s: float = 15.0) -> dict:
    from oracle import optim
    from oracle import ppo as oppo
    from oracle import recurrent as orec

    # the recurrent learner step (env-minibatches, GRU) for recurrent networks
    step = orec.update if w.network.recurrent else oppo.update

    threads = len(os.sched_getaffinity(0))
    rng_w = w
    roll = configs.rollout(rng_w) if w.batch_size * w.network.obs_dim < 6e8 else None
    if roll is None:  # C5: a full-size host rollout is 8.7 GB; sample 1/16 of the envs
        rng_w = w.scaled(num_envs=max(w.num_envs // 16, w.ppo.num_minibatches))
        roll = configs.rollout(rng_w)
    params = init_params(w.network, seed=0, init=w.init)
    perms = configs.permutations(rng_w)
    # GAE + bootstrap alone
    t0 = time.perf_counter()
    step(w.network, w.ppo, w.optimizer, params, optim.init_state(params), roll, perms,
         max_minibatches=0)
    t_gae = time.perf_counter() - t0
    # minibatch steps until the budget is used (at least one)
    mb_ratio = w.minibatch_size / rng_w.minibatch_size
    done, t_mb = 0, 0.0
    while done < w.ppo.update_epochs * w.ppo.num_minibatches:
        t0 = time.perf_counter()
        step(w.network, w.ppo, w.optimizer, params, optim.init_state(params), roll, perms,
             max_minibatches=done + 1)
        t_mb = time.perf_counter() - t0 - t_gae
        done += 1
        if t_mb * 1 > budget_s / 4 or t_mb > budget_s / (done + 1):
            break
    per_mb = max(t_mb, 1e-9) / done * mb_ratio
    t_update = t_gae * (w.batch_size / rng_w.batch_size) + per_mb * w.ppo.update_epochs * w.ppo.num_minibatches
    value = w.batch_size / t_update
    return {"value": value, "unit": "env-steps/s", "cores": threads, "kind": "port",
            "sample": (f"NumPy oracle (float32, BLAS threads={threads}) on the {rng_w.name} "
                       f"rollout T={rng_w.num_steps} N={rng_w.num_envs}: bootstrap+GAE plus {done} "
                       f"of {w.ppo.update_epochs * w.ppo.num_minibatches} minibatch steps "
                       f"(rows scaled x{mb_ratio:g}), extrapolated to one full update")}


def run_reference(args, w):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    steps = []
    cb = None
    for _ in range(args.warmup + args.steps):
        cb = cpu_baseline(w, budget_s=8.0)
        steps.append(cb["value"])
    value = statistics.median(steps[args.warmup:]) if args.steps else steps[-1]
    cb["value"] = value
    line = {
        "impl": "reference", "metric": "ppo_learner_env_steps_per_sec", "value": value,
        "unit": "env-steps/s", "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": 1000.0 * w.batch_size / value, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": w.name, "T": w.num_steps, "N_per_gpu": w.num_envs,
                   "epochs": w.ppo.update_epochs, "minibatches": w.ppo.num_minibatches,
                   "description": w.description},
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
    ap.add_argument("--config", default="c2")
    ap.add_argument("--precision", default=None)
    ap.add_argument("--impl", default="native", choices=["native", "reference"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-profile", action="store_true",
                    help="skip the per-kernel-class profiled pass (for ncu launch lists)")
    args = ap.parse_args()

    kw = {"precision": args.precision} if args.precision else {}
    w = configs.make(args.config, **kw)
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
        "config": {"workload": w.name, "T": w.num_steps, "N_per_gpu": w.num_envs,
                   "epochs": w.ppo.update_epochs, "minibatches": w.ppo.num_minibatches,
                   "minibatch_rows": w.minibatch_size, "precision": w.precision,
                   "parallelism": f"dp{world}", "l2": "inputs larger than L2 (obs rollout "
                   f"{w.batch_size * w.network.obs_dim * 4 / 1e6:.0f} MB per GPU)",
                   "description": w.description},
        "roofline": roof,
        "gae_hbm_gbs": gae_bw["gbs"],
        "gae": gae_bw,
        "kernel_ms_per_step": {k: v[0] for k, v in sorted(prof.items())},
        "gpu_launches": int(launches),
        "clocks": clocks.summary(),
        "e2e": e2e,
    }
    if world == 1 and not args.no_cpu_baseline:
        line["cpu_baseline"] = cpu_baseline(w)
    print(json.dumps(line), flush=True)
    if world > 1:
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
