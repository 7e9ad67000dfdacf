"""PPOState as the reference's pytree and its msgpack checkpoint, on the CPU: the tree has the
optax chain shape (EmptyState, ScaleByAdamState(count, mu, nu), EmptyState), mu / nu / params
nest by the layout's names, and save -> load gives back the same state bit for bit."""
import numpy as np
import torch

from boonta_b200 import checkpoint, configs
from boonta_b200.ppo import AdamState, PPOState
from boonta_b200.spec import init_params, param_layout


def _state(w, seed=0):
    layout = param_layout(w.network)
    rng = np.random.default_rng(seed)
    p = torch.as_tensor(layout.flatten(init_params(w.network, seed=seed, init=w.init)))
    # moments on the named entries (the alignment gaps between groups are not state)
    flat = lambda x: torch.as_tensor(layout.flatten(layout.unflatten(x.astype(np.float32))))
    mu = flat(rng.standard_normal(layout.total))
    nu = flat(rng.random(layout.total))
    return layout, PPOState(step=torch.tensor(7, dtype=torch.int64), params=p,
                            optimizer_state=AdamState(mu, nu, torch.tensor(48, dtype=torch.int32)))


def test_state_pytree_has_the_optax_chain_shape():
    w = configs.c1()
    layout, st = _state(w)
    tree = checkpoint.state_pytree(st, layout)
    assert set(tree) == {"step", "params", "optimizer_state"}
    chain = tree["optimizer_state"]
    assert len(chain) == 3 and type(chain[0]).__name__ == "EmptyState"
    assert type(chain[1]).__name__ == "ScaleByAdamState" and chain[1].count == 48
    assert set(tree["params"]) == set(chain[1].mu) == set(chain[1].nu)
    np.testing.assert_array_equal(tree["params"]["torso"]["0"]["kernel"],
                                  layout.unflatten(st.params.numpy())["torso/0/kernel"])


def test_state_dict_encoding_keys_tuples_by_position():
    w = configs.c1()
    layout, st = _state(w)
    sd = checkpoint.to_state_dict(checkpoint.state_pytree(st, layout))
    assert set(sd["optimizer_state"]) == {"0", "1", "2"}
    assert sd["optimizer_state"]["0"] == {} and set(sd["optimizer_state"]["1"]) == {"count", "mu", "nu"}


def test_checkpoint_round_trip_is_exact(tmp_path):
    for name in ("c1", "c4"):
        w = configs.make(name)
        layout, st = _state(w, seed=3)
        path = checkpoint.save(tmp_path / f"{name}.msgpack", st, layout)
        back = checkpoint.load(path, layout, device="cpu")
        assert int(back.step) == 7 and int(back.optimizer_state.count) == 48
        assert torch.equal(back.params, st.params)
        assert torch.equal(back.optimizer_state.mu, st.optimizer_state.mu)
        assert torch.equal(back.optimizer_state.nu, st.optimizer_state.nu)
