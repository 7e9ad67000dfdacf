"""The multi-GPU gradient rule on CPU ranks (gloo, world size 2): every rank sums the loss
gradient of its own rows of each *global* minibatch, scaled by 1 / global minibatch size;
one all-reduce then equals the single-process gradient of that minibatch
(boonta/algorithms/ppo.py:148-200 with the batch sharded on envs)."""
import os

import numpy as np
import pytest

from boonta_b200 import configs
from boonta_b200.sharding import local_rows
from boonta_b200.spec import init_params


def _workload():
    return configs.c2(precision="fp32").scaled(num_steps=4, num_envs=16, num_minibatches=4,
                                               update_epochs=1)


def _global_rollout(w, world):
    rolls = [configs.rollout(w, seed=10 + r) for r in range(world)]
    out = {}
    for k in rolls[0]:
        axis = 0 if k == "bootstrap_obs" else 1
        out[k] = np.concatenate([r[k] for r in rolls], axis=axis)
    return rolls, out


def _minibatch(roll, idx, adv, ret):
    t, n = roll["reward"].shape
    b = t * n
    return {
        "obs": roll["obs"].reshape(b, -1)[idx],
        "action": roll["action"].reshape(b, *roll["action"].shape[2:])[idx],
        "log_prob": roll["log_prob"].reshape(b)[idx],
        "value": roll["value"].reshape(b)[idx],
        "advantages": adv.reshape(b)[idx],
        "returns": ret.reshape(b)[idx],
    }


def _rank_main(rank, world, port, q):
    import torch
    import torch.distributed as dist

    from oracle import ppo as oppo

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    w = _workload()
    rolls, _ = _global_rollout(w, world)
    roll = rolls[rank]
    params = {k: v.astype(np.float64) for k, v in init_params(w.network, seed=0).items()}
    rng = np.random.default_rng(5)
    t, n = roll["reward"].shape
    adv_g = rng.standard_normal((t, n * world))
    ret_g = rng.standard_normal((t, n * world))
    adv = adv_g[:, rank * n:(rank + 1) * n]
    ret = ret_g[:, rank * n:(rank + 1) * n]
    perm = np.random.default_rng(9).permutation(t * n * world)
    mb_global = len(perm) // w.ppo.num_minibatches
    idx = local_rows(perm[:mb_global], rank, n, world)
    mb = _minibatch(roll, idx, adv, ret)
    # gradient of the rank's rows with the global 1/mb: loss_and_grads scales by 1/len(rows)
    _, _, grads = oppo.loss_and_grads(w.network, w.ppo, params, mb, dtype=np.float64)
    scale = len(idx) / mb_global
    flat = np.concatenate([grads[k].ravel() * scale for k in sorted(grads)])
    buf = torch.from_numpy(flat)
    dist.all_reduce(buf)
    q.put((rank, buf.numpy()))
    dist.destroy_process_group()


def test_sharded_gradient_sum_equals_the_global_minibatch_gradient():
    import multiprocessing as mp
    import socket

    from oracle import ppo as oppo

    world = 2
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_rank_main, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    results = dict(q.get(timeout=120) for _ in range(world))
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    np.testing.assert_array_equal(results[0], results[1])  # identical bytes on every rank

    w = _workload()
    _, roll = _global_rollout(w, world)
    params = {k: v.astype(np.float64) for k, v in init_params(w.network, seed=0).items()}
    rng = np.random.default_rng(5)
    t, n = roll["reward"].shape
    adv, ret = rng.standard_normal((t, n)), rng.standard_normal((t, n))
    perm = np.random.default_rng(9).permutation(t * n)
    mb_global = len(perm) // w.ppo.num_minibatches
    _, _, grads = oppo.loss_and_grads(w.network, w.ppo, params,
                                      _minibatch(roll, perm[:mb_global], adv, ret), dtype=np.float64)
    ref = np.concatenate([grads[k].ravel() for k in sorted(grads)])
    np.testing.assert_allclose(results[0], ref, rtol=1e-10, atol=1e-13)


def test_local_rows_partition_a_global_minibatch():
    world, n, t = 4, 8, 5
    perm = np.random.default_rng(0).permutation(t * n * world)
    seen = []
    for r in range(world):
        loc = local_rows(perm, r, n, world)
        tt, nn = np.divmod(loc, n)
        seen.extend((tt * n * world + r * n + nn).tolist())
    assert sorted(seen) == sorted(perm.tolist())
