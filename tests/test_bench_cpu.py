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


def test_batched_workloads_match_configs_1_and_3():
    """frames8 = config 1 (8 periodic frames of 96 atoms in a 10 A box, ictd C 32, 2 layers,
    8 bessel); mol256 = config 3 (256 molecules of 10-30 atoms, o3 C 64, 3 layers, one field
    vector per molecule)."""
    w = bench.WORKLOADS["frames8"]
    s = bench.batched_system(w)
    assert s["pos"].shape == (8 * 96, 3) and s["cell"].shape == (8, 3, 3) and tuple(s["pbc"]) == (True,) * 3
    assert len(set(s["Z"].tolist())) == 3
    cfg = bench.model_cfg(w)
    assert (cfg.channels, cfg.num_interaction, cfg.function_type, cfg.o3) == (32, 2, "bessel", False)
    assert list(s["frame_ptr"]) == list(range(0, 8 * 96 + 1, 96))
    w = bench.WORKLOADS["mol256"]
    s = bench.batched_system(w)
    sizes = s["frame_ptr"][1:] - s["frame_ptr"][:-1]
    assert len(sizes) == 256 and sizes.min() >= 10 and sizes.max() <= 30 and s["field"].shape == (256, 3)
    cfg = bench.model_cfg(w)
    assert (cfg.channels, cfg.num_interaction, cfg.o3) == (64, 3, True)
    sd = bench.seeded_weights(cfg)
    assert any(k.startswith("physical_tensor_heads.") for k in sd)


def test_fp32_context_uses_the_measured_peak():
    roof = {"bound": "hbm", "algorithmic_tflops": 20.0}
    ctx = bench.fp32_context(roof, {"sm_mhz": 1965.0}, measured={"tflops": 80.0, "how": "probe"})
    assert ctx["peak_tflops"] == 80.0 and ctx["frac"] == 0.25 and ctx["peak_source"] == "measured: probe"
    assert ctx["nominal_tflops"] == pytest.approx(148 * 128 * 2 * 1965e6 / 1e12)


def test_clock_records_of_several_gpus_combine_conservatively():
    one = {"sm_mhz": 1950.0, "sm_max_mhz": 1965.0, "reasons": ["sw_power_cap"], "samples": 6}
    assert bench.combine_clocks([one]) is one
    two = {"sm_mhz": 1792.5, "sm_max_mhz": 1965.0, "reasons": ["hw_slowdown", "sw_power_cap"], "samples": 5}
    none = {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no samples"]}
    c = bench.combine_clocks([one, two, none])
    assert c["sm_mhz"] == 1792.5 and c["sm_max_mhz"] == 1965.0
    assert c["reasons"] == ["hw_slowdown", "no samples", "sw_power_cap"]
    assert c["samples"] == 11 and [r["sm_mhz"] for r in c["per_rank"]] == [1950.0, 1792.5, None]


def test_each_rank_writes_its_own_clock_file():
    assert bench.rank_path(None, 3, 8) is None
    assert bench.rank_path("/tmp/c.csv", 0, 1) == "/tmp/c.csv"
    assert bench.rank_path("/tmp/c.csv", 3, 8) == "/tmp/c_rank3.csv"
    assert bench.rank_path("/tmp/c", 1, 2) == "/tmp/c_rank1.csv"
