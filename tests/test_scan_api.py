"""Host-side checks of boonta_b200.scan (the SSM scan's Python surface) that need no GPU: the
implementation registry mirrors the reference's (boonta/networks/kernels/__init__.py:12-19) and
the torch reference forms agree with the oracle's restatements."""
import numpy as np
import pytest
import torch

from boonta_b200 import scan as bscan
from oracle import scan as osc


def _problem(seed, shape=(3, 10, 6)):
    rng = np.random.default_rng(seed)
    a = (rng.uniform(size=shape) * 0.9 + 0.05).astype(np.float32)
    b = rng.uniform(size=shape).astype(np.float32)
    init = rng.standard_normal((shape[0], shape[2])).astype(np.float32)
    return a, b, init


def test_registry_names_and_default():
    assert bscan.get_scan_implementation() is bscan.scan
    assert set(bscan.IMPLEMENTATIONS) == {"cuda", "sequential", "associative"}
    with pytest.raises(KeyError):
        bscan.get_scan_implementation("pallas")


def test_torch_reference_forms_match_the_oracle():
    a, b, init = _problem(1)
    t = lambda x: torch.from_numpy(x)
    seq = bscan.sequential(t(a), t(b), t(init)).numpy()
    np.testing.assert_allclose(seq, osc.sequential(a, b, init), rtol=1e-6, atol=1e-6)
    assoc = bscan.associative(t(a), t(b), t(init)).numpy()
    np.testing.assert_allclose(assoc, osc.exact(a, b, init), rtol=1e-5, atol=1e-5)


def test_the_native_scan_rejects_host_tensors():
    a, b, init = _problem(2)
    with pytest.raises(ValueError, match="CUDA"):
        bscan.scan(torch.from_numpy(a), torch.from_numpy(b), torch.from_numpy(init))
