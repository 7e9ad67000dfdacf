"""CUDA-graph replay of the learner update: bit-identical to eager execution.

bt_learner_update runs its first call with a given set of batch pointers eagerly, captures
the second into a CUDA graph and replays it afterwards; permutations and statistics pass
through internal buffers, so they may change between replays.
"""
import numpy as np
import pytest

from boonta_b200 import configs

pytestmark = pytest.mark.gpu


def _run(w, graphs: bool, steps: int):
    import torch

    from boonta_b200.learner import Learner, to_device
    from boonta_b200.spec import init_params

    lrn = Learner.from_workload(w)
    lrn.use_graphs(graphs)
    lrn.set_state(init_params(w.network, seed=3))
    roll = to_device(configs.rollout(w, seed=5))
    stats = []
    for i in range(steps):
        perms = torch.as_tensor(configs.permutations(w, seed=11 + i))  # a new tensor each step
        stats.append(lrn.update(roll, perms).cpu().numpy())
    params, mu, nu, count = lrn.get_state()
    return (params.cpu().numpy(), mu.cpu().numpy(), nu.cpu().numpy(), count,
            np.stack(stats), lrn.launch_count())


CASES = {
    "c2_fp32": lambda: configs.make("c2", precision="fp32").scaled(
        num_steps=8, num_envs=256, num_minibatches=4, update_epochs=2),
    "c2_bf16x3": lambda: configs.make("c2", precision="bf16x3").scaled(
        num_steps=8, num_envs=256, num_minibatches=4, update_epochs=2),
    "c4_gru": lambda: configs.make("c4").scaled(num_steps=8, num_envs=32, num_minibatches=2,
                                                update_epochs=2),
}


@pytest.mark.parametrize("name", list(CASES))
def test_graph_replay_matches_eager_updates(name):
    w = CASES[name]()
    eager = _run(w, graphs=False, steps=4)
    graph = _run(w, graphs=True, steps=4)  # eager, capture + replay, replay, replay
    for a, b in zip(eager[:3], graph[:3]):
        np.testing.assert_array_equal(a, b)
    assert eager[3] == graph[3] == 4 * w.ppo.update_epochs * w.ppo.num_minibatches
    np.testing.assert_array_equal(eager[4], graph[4])
    assert eager[5] == graph[5]  # replays count the graph's kernels as launches
