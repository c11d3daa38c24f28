"""bench.py's workload table and work model on CPU: the sparse workloads carry BASELINE configs 2
and 5, and the per-stage algorithmic work matches the hot path's per-unit figures."""

import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)

import bench  # noqa: E402


def test_sparse_component_counts():
    assert bench.sparse_comps(2) == 34   # (0,0,0) (0,1,1) (0,2,2) (1,0,1) (1,1,2) (2,0,2): 1+3+9+3+9+9
    assert bench.sparse_comps(3) == 142


def test_workloads_match_the_baseline_configs():
    w = bench.WORKLOADS["water3k"]
    assert (w["model"], w["channels"], w["lmax"], w["num_interaction"]) == ("sparse", 64, 2, 3)
    assert 3 * w["n_side"] ** 3 == 3000 and w["box"] == 31.0
    for name, atoms in (("fcc32k", 32000), ("fcc250k", 250000)):
        w = bench.WORKLOADS[name]
        assert (w["model"], w["channels"], w["lmax"], w["num_interaction"]) == ("sparse", 128, 3, 3)
        assert 4 * w["cells"][0] * w["cells"][1] * w["cells"][2] == atoms
    w = bench.WORKLOADS["si1m"]
    assert (w["model"], w["channels"], w["num_interaction"]) == ("ictd", 64, 3)
    assert 8 * w["cells"][0] * w["cells"][1] * w["cells"][2] == 1_000_000


@pytest.mark.parametrize("lmax,C", [(2, 64), (3, 128)])
def test_sparse_stage_work(lmax, C):
    cfg = bench.sparse_cfg(dict(channels=C, lmax=lmax, num_interaction=3, max_atomvalue=30))
    N, E = 1000, 45000
    fwd_flops, fwd_bytes = bench.algorithmic_work("sparse_conv2_forward", N, E, cfg)
    bwd_flops, bwd_bytes = bench.algorithmic_work("sparse_conv2_backward", N, E, cfg)
    K3 = bench.sparse_comps(lmax)
    edge = 2.0 * E * 65 * C * K3
    node = 2.0 * N * K3 * 65 * C * C
    assert fwd_flops == pytest.approx(edge + node)
    assert bwd_flops == pytest.approx(2 * edge + node)
    assert fwd_bytes > 0 and bwd_bytes > fwd_bytes
    assert bench.algorithmic_work("sparse_readout_gram_forward", N, E, cfg) is None


def test_fp32_context():
    roof = {"bound": "hbm", "algorithmic_tflops": 17.08}
    ctx = bench.fp32_context(roof, {"sm_mhz": 1965.0})
    assert ctx["peak_tflops"] == pytest.approx(148 * 128 * 2 * 1965e6 / 1e12)
    assert ctx["frac"] == pytest.approx(17.08 / ctx["peak_tflops"])
    assert bench.fp32_context(roof, {"sm_mhz": None, "reasons": ["no samples"]})["sm_mhz"] == 1965.0
    assert bench.fp32_context({"bound": "tensor", "algorithmic_tflops": 300.0}, {"sm_mhz": 1965.0}) is None
    assert bench.fp32_context(None, None) is None
