"""Failure detection on the GPU without a fault: a bounded wait that nothing satisfies, and the
GRU sequence kernels' grid-wide step barrier with an unreachable target, give up after their
limits, report BT_ERR_TIMEOUT, and leave the context usable; a learner's device-side error word
reads clean after normal updates."""
import time

import numpy as np
import pytest

from boonta_b200 import _lib, configs

pytestmark = pytest.mark.gpu


def test_bounded_wait_gives_up_and_the_context_stays_usable():
    import torch

    from boonta_b200.learner import Learner, to_device

    s = torch.cuda.current_stream().cuda_stream
    t0 = time.perf_counter()
    rc = _lib.lib().bt_selftest_bounded_wait(50_000, s)  # 50 ms limit
    dt = time.perf_counter() - t0
    assert rc == _lib.BT_ERR_TIMEOUT
    assert b"gave up" in _lib.lib().bt_last_error()
    assert 0.04 <= dt < 5.0
    # the context still works: a learner update runs and reports no device-side failure
    w = configs.make("c2", precision="bf16x3").scaled(num_steps=8, num_envs=128,
                                                      num_minibatches=2, update_epochs=1)
    lrn = Learner.from_workload(w)
    from boonta_b200.spec import init_params

    lrn.set_state(init_params(w.network, seed=0))
    st = lrn.update(to_device(configs.rollout(w)), torch.as_tensor(configs.permutations(w)))
    lrn.check()
    assert np.isfinite(st.cpu().numpy()).all()


def test_selftest_rejects_limits_outside_the_bound():
    import torch

    s = torch.cuda.current_stream().cuda_stream
    assert _lib.lib().bt_selftest_bounded_wait(0, s) == _lib.BT_ERR_INVALID
    assert _lib.lib().bt_selftest_bounded_wait(3_000_000, s) == _lib.BT_ERR_INVALID


def test_gru_step_barrier_gives_up_and_the_context_stays_usable():
    import torch

    from boonta_b200.learner import Learner, to_device
    from boonta_b200.spec import init_params

    s = torch.cuda.current_stream().cuda_stream
    t0 = time.perf_counter()
    rc = _lib.lib().bt_selftest_gru_barrier(50_000, s)  # 50 ms limit, 4 CTAs
    dt = time.perf_counter() - t0
    assert rc == _lib.BT_ERR_TIMEOUT
    assert b"barrier gave up" in _lib.lib().bt_last_error()
    assert 0.04 <= dt < 5.0
    assert _lib.lib().bt_selftest_gru_barrier(0, s) == _lib.BT_ERR_INVALID
    # the context still works: a recurrent update (the same sequence kernels) runs clean
    w = configs.c4().scaled(num_steps=8, num_envs=32, num_minibatches=2, update_epochs=1)
    lrn = Learner.from_workload(w)
    lrn.set_state(init_params(w.network, seed=0))
    st = lrn.update(to_device(configs.rollout(w)), torch.as_tensor(configs.permutations(w)))
    lrn.check()
    assert np.isfinite(st.cpu().numpy()).all()
