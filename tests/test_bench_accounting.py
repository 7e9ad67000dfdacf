"""The work accounting behind bench.py's roofline line, on the CPU: the algorithmic FLOPs per
env-step of each workload against the per-sample derivation (forward = sum of K*N over the
layers, backward = dW (as forward) + dX (every layer but the first), times the epochs; the
bench also counts the bias column and the head products), the GAE byte count, and the
roofline arithmetic (bound, achieved, fraction) on a made-up per-class profile."""
import pytest

import bench
from boonta_b200 import configs

# MFLOP per env-step: 2 x MACs per sample per epoch x epochs (+ the bootstrap forward)
EXPECTED_MFLOP = {"c1": 0.1071, "c2": 7.07, "c3": 5.87, "c4": 4.89, "c5": 81.0}


@pytest.mark.parametrize("name", sorted(EXPECTED_MFLOP))
def test_algorithmic_flops_per_env_step(name):
    w = configs.make(name)
    work = bench.class_work(w)
    flops = sum(f for f, _ in work.values())
    assert flops / w.batch_size / 1e6 == pytest.approx(EXPECTED_MFLOP[name], rel=0.03)


def test_gae_bytes_are_eighteen_per_env_step_plus_the_bootstrap():
    w = configs.make("c2")
    assert bench.gae_bytes(w) == 18 * 64 * 8192 + 4 * 8192


def test_roofline_picks_the_longer_bound_and_reports_the_fraction():
    w = configs.make("c5")
    work = bench.class_work(w)
    peaks = {"hbm_gbs": 6558.4, "bf16_tflops": 1650.1, "bf16_tflops_sustained": 1377.9}
    flops, nbytes = work["gemm_dw"]
    prof = {"gemm_dw": (20.0, 192), "gemm_fwd": (5.0, 195)}  # ms per update, launches
    line = bench.roofline(w, prof, peaks, "measured")
    assert line["kernel"] == "gemm_dw" and line["launches"] == 192
    tensor_s, hbm_s = flops / 1377.9e12, nbytes / 6558.4e9
    assert line["bound"] == ("tensor" if tensor_s >= hbm_s else "hbm")
    if line["bound"] == "tensor":
        assert line["achieved"] == pytest.approx(flops / 0.020 / 1e12)
        assert line["frac"] == pytest.approx(line["achieved"] / 1377.9)
    else:
        assert line["achieved"] == pytest.approx(nbytes / 0.020 / 1e9)
        assert line["frac"] == pytest.approx(line["achieved"] / 6558.4)
