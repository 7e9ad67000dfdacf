"""Multi-GPU learner on 2 GPUs (BT_TEST_WORLD=N for another rank count), one process per GPU:
the NVLink peer-memory gradient exchange fused with the optimizer step (and, for one case, the
NCCL all-reduce path); the ranks end bitwise identical and equal to the single-process oracle
update of the global batch (global permutation, boonta/algorithms/ppo.py:200). Skipped with
fewer GPUs than ranks."""
import dataclasses
import os

import numpy as np
import pytest

from boonta_b200 import configs
from boonta_b200.spec import init_params

pytestmark = pytest.mark.gpu

WORLD = int(os.environ.get("BT_TEST_WORLD", "2"))


def _workload(kind):
    if kind == "c4":
        return configs.c4().scaled(num_steps=8, num_envs=32, num_minibatches=4, update_epochs=2)
    if kind == "fp32_nccl":
        return _workload("fp32")
    if kind == "fp32_norm":
        # advantage normalisation over the global batch: the moments are summed across ranks
        # (boonta/algorithms/ppo.py:220-221 over the sharded [T, N_global] advantages)
        w = _workload("fp32")
        return dataclasses.replace(w, ppo=dataclasses.replace(w.ppo, normalize_advantage=True))
    if kind == "bf16":
        # C5's network and arithmetic (bf16 GEMMs, the bf16 rollout copy) on a small rollout
        return configs.c5().scaled(num_steps=8, num_envs=64, num_minibatches=4, update_epochs=2)
    return configs.c2(precision=kind).scaled(num_steps=8, num_envs=64, num_minibatches=4,
                                             update_epochs=2)


def _rollouts(w):
    return [configs.rollout(w, seed=20 + r) for r in range(WORLD)]


def _rank_main(rank, port, kind, q):
    import datetime

    import torch
    import torch.distributed as dist

    from boonta_b200.learner import Learner, to_device

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=WORLD,
                            timeout=datetime.timedelta(seconds=60))
    torch.cuda.set_device(rank)
    w = _workload(kind)
    lrn = Learner.from_workload(w, world_size=WORLD, rank=rank)
    uid = [Learner.nccl_unique_id() if rank == 0 else None]
    dist.broadcast_object_list(uid, src=0)
    lrn.comm_init(uid[0])
    if kind == "fp32_nccl":
        lrn.use_p2p(False)  # the NCCL all-reduce path instead of the NVLink exchange
    lrn.set_state(init_params(w.network, seed=0, init=w.init))
    roll = _rollouts(w)[rank]
    perms = configs.permutations(w, num_ranks=WORLD)
    st = lrn.update(to_device(roll), torch.as_tensor(perms))
    torch.cuda.synchronize()
    p_, mu, nu, _ = lrn.get_state()
    q.put((rank, p_.cpu().numpy(), st.cpu().numpy(), mu.cpu().numpy(), nu.cpu().numpy()))
    lrn.close()
    dist.destroy_process_group()


def _global(w):
    rolls = _rollouts(w)
    out = {}
    for k in rolls[0]:
        axis = 0 if (k in ("bootstrap_obs", "carry", "last_carry") or rolls[0][k].ndim == 1) else 1
        out[k] = np.concatenate([r[k] for r in rolls], axis=axis)
    return out


@pytest.mark.parametrize("kind", ["fp32", "bf16x3", "c4", "fp32_norm", "fp32_nccl", "bf16"])
def test_two_gpu_update_matches_the_global_oracle(kind):
    import multiprocessing as mp
    import socket

    import torch

    from oracle import optim, recurrent
    from oracle import ppo as oppo

    if torch.cuda.device_count() < WORLD:
        pytest.skip("needs 2 GPUs")
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_rank_main, args=(r, port, kind, q)) for r in range(WORLD)]
    for p in procs:
        p.start()
    res = {}
    for _ in range(WORLD):
        r, params, stats, mu, nu = q.get(timeout=300)
        res[r] = (params, stats, mu, nu)
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    np.testing.assert_array_equal(res[0][0], res[1][0])  # replicas stay bitwise equal
    np.testing.assert_array_equal(res[0][1], res[1][1])
    np.testing.assert_array_equal(res[0][2], res[1][2])  # Adam's moments replicated too
    np.testing.assert_array_equal(res[0][3], res[1][3])

    w = _workload(kind)
    params = init_params(w.network, seed=0, init=w.init)
    roll = _global(w)
    perms = configs.permutations(w, num_ranks=WORLD)
    gw = w.scaled(num_envs=w.num_envs * WORLD)
    if kind == "c4":
        op, _, ostats, _ = recurrent.update(gw.network, gw.ppo, gw.optimizer, params,
                                            optim.init_state(params), roll, perms)
    elif kind == "bf16":
        from _parity import check_params

        from boonta_b200.spec import param_layout

        op64, _, _, _ = oppo.update(gw.network, gw.ppo, gw.optimizer, params,
                                    optim.init_state(params, np.float64), roll, perms,
                                    precision="bf16", dtype=np.float64)
        op32, _, ostats, _ = oppo.update(gw.network, gw.ppo, gw.optimizer, params,
                                         optim.init_state(params), roll, perms, precision="bf16")
        got = param_layout(w.network).unflatten(res[0][0])
        bad = check_params("2-GPU bf16", "bf16", params, got, op64, op32,
                           w.ppo.update_epochs * w.ppo.num_minibatches, w.optimizer.lr)
        assert not bad, bad
        return
    else:
        op, _, ostats, _ = oppo.update(gw.network, gw.ppo, gw.optimizer, params,
                                       optim.init_state(params), roll, perms)
    from boonta_b200.spec import param_layout

    got = param_layout(w.network).unflatten(res[0][0])
    steps = w.ppo.update_epochs * w.ppo.num_minibatches
    for k in op:
        # Zero-initialised tensors (biases) have no magnitude of their own: their error is
        # measured against the largest move Adam can make in `steps` steps. With split-bf16
        # products a bias whose gradient sum nearly cancels can land a few percent of that
        # move away (the per-minibatch gradients themselves agree within 1e-4).
        floor = steps * w.optimizer.lr * np.sqrt(op[k].size)
        rel = np.linalg.norm(got[k] - op[k]) / max(np.linalg.norm(op[k]), floor)
        bound = 1e-3 if (kind != "bf16x3" or np.any(params[k] != 0)) else 5e-2
        assert rel <= bound, (k, rel)
    np.testing.assert_allclose(res[0][1], ostats, rtol=2e-3, atol=2e-4)
