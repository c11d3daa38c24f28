"""GPU parity of the native pure-cartesian-ictd E + F + stress against the reference."""

import numpy as np
import pytest
import torch

import gpu_util as U

pytestmark = [pytest.mark.gpu, U.needs_gpu]


@pytest.mark.parametrize("tag", ["a", "b", "c", "e", "z"])
def test_energy_forces_stress_match_reference(tag):
    eng, g, (pos, Z, batch, cell), c, _, _ = U.golden_engine(tag)
    out = eng.energy_forces(pos, Z, batch, cell, g)
    torch.cuda.synchronize()
    assert eng.status() == 0
    E = out["energy"].cpu().numpy()
    F = out["forces"].cpu().numpy()
    S = out["stress"].cpu().numpy()
    assert np.all(np.abs(E - c["ref64_energy"]) <= U.E_RTOL * np.abs(c["ref64_energy"])), (E, c["ref64_energy"])
    assert U.rel_max(F, c["ref64_forces"]) <= U.F_RTOL, U.rel_max(F, c["ref64_forces"])
    assert U.rel_max(S, c["ref64_stress"]) <= U.S_RTOL, U.rel_max(S, c["ref64_stress"])
    np.testing.assert_allclose(out["atom_energy"].cpu().numpy(), c["ref64_atom_energy"], rtol=1e-4, atol=1e-4)


def test_forces_sum_to_zero_and_repeatable():
    eng, g, (pos, Z, batch, cell), c, _, _ = U.golden_engine("a")
    o1 = eng.energy_forces(pos, Z, batch, cell, g)
    o2 = eng.energy_forces(pos, Z, batch, cell, g)
    torch.cuda.synchronize()
    F = o1["forces"].double()
    assert F.sum(0).abs().max().item() < 1e-3 * F.abs().max().item()
    assert torch.equal(o1["forces"], o2["forces"]) and torch.equal(o1["energy"], o2["energy"])


def test_energy_weights_ghost_convention():
    """num_local excludes trailing atoms from E; forces still act on them (LAMMPS convention)."""
    eng, g, (pos, Z, batch, cell), c, _, _ = U.golden_engine("b")
    n = pos.shape[0]
    full = eng.energy_forces(pos, Z, batch, cell, g)
    part = eng.energy_forces(pos, Z, batch, cell, g, num_local=n // 2)
    ae = full["atom_energy"].double()
    torch.cuda.synchronize()
    assert abs(part["energy"].item() - ae[: n // 2].sum().item()) < 1e-4 * abs(ae[: n // 2].sum().item()) + 1e-5


@pytest.mark.parametrize("tag,n_cells", [("c", (5, 5, 3)), ("b", (3, 3, 5))])
def test_tensor_core_readout_matches_cuda_core_readout(tag, n_cells):
    """tcgen05 readout (default) vs the CUDA-core readout on several 128-node tiles (partial last tile)."""
    from fsctep_b200 import _native as NAT
    from fsctep_b200 import systems
    from fsctep_b200.neighbors import build_graph

    eng, _, _, c, icfg, sd = U.golden_engine(tag)
    s = systems.diamond_crystal(n_cells=n_cells, seed=21)
    dev = torch.device("cuda")
    pos, cell = torch.tensor(s["pos"], device=dev), torch.tensor(s["cell"], device=dev)
    g = build_graph(pos, cell, 5.0)
    Z, b = torch.tensor(s["Z"], device=dev), torch.tensor(s["batch"], device=dev)
    try:
        NAT.lib().fsc_ictd_set_readout_path(1)
        ref = eng.energy_forces(pos, Z, b, cell, g)
        torch.cuda.synchronize()
        NAT.lib().fsc_ictd_set_readout_path(0)
        out = eng.energy_forces(pos, Z, b, cell, g)
        torch.cuda.synchronize()
        assert eng.status() == 0
    finally:
        NAT.lib().fsc_ictd_set_readout_path(0)
    assert pos.shape[0] % 128 != 0
    e, er = out["energy"].double().cpu(), ref["energy"].double().cpu()
    assert (e - er).abs().max().item() <= 1e-5 * er.abs().max().item(), (e, er)
    assert U.rel_max(out["forces"].cpu().numpy(), ref["forces"].cpu().numpy()) <= 1e-4
    assert U.rel_max(out["atom_energy"].cpu().numpy(), ref["atom_energy"].cpu().numpy()) <= 1e-4


@pytest.mark.parametrize("nb,kind,n_cells", [(8, "gaussian", (3, 3, 3)), (12, "bessel", (5, 3, 3))])
def test_tensor_core_radial_matches_cuda_core(nb, kind, n_cells):
    """tcgen05 radial MLPs (default) vs the CUDA-core ones; nb=12 exercises the 16-wide padded basis."""
    from fsctep_b200 import _native as NAT
    from fsctep_b200 import systems
    from fsctep_b200.ictd import ICTDConfig, ICTDEngine
    from fsctep_b200.models import reference_state_dict_shapes
    from fsctep_b200.neighbors import build_graph
    from fsctep_b200.weights import seeded_state_dict

    cfg = ICTDConfig(channels=32, num_interaction=3, number_of_basis=nb, max_radius=5.0, function_type=kind,
                     max_atomvalue=16)
    eng = ICTDEngine(seeded_state_dict(reference_state_dict_shapes(cfg), 5), cfg, "cuda")
    s = systems.diamond_crystal(n_cells=n_cells, seed=23)
    dev = torch.device("cuda")
    pos, cell = torch.tensor(s["pos"], device=dev), torch.tensor(s["cell"], device=dev)
    g = build_graph(pos, cell, 5.0)
    assert g.num_edges % 128 != 0
    Z, b = torch.tensor(s["Z"], device=dev), torch.tensor(s["batch"], device=dev)
    try:
        NAT.lib().fsc_ictd_set_radial_path(1)
        ref = eng.energy_forces(pos, Z, b, cell, g)
        torch.cuda.synchronize()
        NAT.lib().fsc_ictd_set_radial_path(0)
        out = eng.energy_forces(pos, Z, b, cell, g)
        torch.cuda.synchronize()
        assert eng.status() == 0
    finally:
        NAT.lib().fsc_ictd_set_radial_path(0)
    e, er = out["energy"].double().cpu(), ref["energy"].double().cpu()
    assert (e - er).abs().max().item() <= 1e-5 * er.abs().max().item(), (e, er)
    assert U.rel_max(out["forces"].cpu().numpy(), ref["forces"].cpu().numpy()) <= 1e-4
    assert U.rel_max(out["stress"].cpu().numpy(), ref["stress"].cpu().numpy()) <= 1e-4


@pytest.mark.parametrize("channels,n_cells", [(64, (5, 3, 3)), (32, (3, 3, 5))])
def test_tensor_core_gemms_match_cuda_core(channels, n_cells):
    """tcgen05 channel-mixing / MainNet GEMMs (default) vs the CUDA-core GEMM: node counts that
    leave partial 128-row tiles for every component count R (1, 3, 5), and N < tile width (C = 32)."""
    from fsctep_b200 import _native as NAT
    from fsctep_b200 import systems
    from fsctep_b200.ictd import ICTDConfig, ICTDEngine
    from fsctep_b200.models import reference_state_dict_shapes
    from fsctep_b200.neighbors import build_graph
    from fsctep_b200.weights import seeded_state_dict

    cfg = ICTDConfig(channels=channels, num_interaction=3, number_of_basis=8, max_radius=5.0,
                     function_type="gaussian", max_atomvalue=16)
    eng = ICTDEngine(seeded_state_dict(reference_state_dict_shapes(cfg), 9), cfg, "cuda")
    s = systems.diamond_crystal(n_cells=n_cells, seed=27)
    dev = torch.device("cuda")
    pos, cell = torch.tensor(s["pos"], device=dev), torch.tensor(s["cell"], device=dev)
    g = build_graph(pos, cell, 5.0)
    Z, b = torch.tensor(s["Z"], device=dev), torch.tensor(s["batch"], device=dev)
    assert pos.shape[0] % 125 and pos.shape[0] % 126 and pos.shape[0] % 128
    try:
        NAT.lib().fsc_ictd_set_gemm_path(1)
        ref = eng.energy_forces(pos, Z, b, cell, g)
        torch.cuda.synchronize()
        NAT.lib().fsc_ictd_set_gemm_path(0)
        out = eng.energy_forces(pos, Z, b, cell, g)
        torch.cuda.synchronize()
        assert eng.status() == 0
    finally:
        NAT.lib().fsc_ictd_set_gemm_path(0)
    e, er = out["energy"].double().cpu(), ref["energy"].double().cpu()
    assert (e - er).abs().max().item() <= 1e-5 * er.abs().max().item(), (e, er)
    assert U.rel_max(out["forces"].cpu().numpy(), ref["forces"].cpu().numpy()) <= 1e-4
    assert U.rel_max(out["atom_energy"].cpu().numpy(), ref["atom_energy"].cpu().numpy()) <= 1e-4
    assert U.rel_max(out["stress"].cpu().numpy(), ref["stress"].cpu().numpy()) <= 1e-4


@pytest.mark.parametrize("channels,kind", [(64, "diamond"), (32, "diamond"), (64, "frames")])
def test_tensor_core_conv2_gates_match_cuda_core(channels, kind):
    """tcgen05 conv2 gate / harmonic gradients (conv2 path 1; 14 edges of a receiver per
    128 x 48 product) vs the CUDA-core kernel (the default): degrees of 28 (two full tiles) and
    of 30-70 (partial tiles).  Energies are the same bits (forward unchanged); forces and stress
    agree to fp32 accuracy; the tensor-core reverse pass repeats bit for bit."""
    from fsctep_b200 import _native as NAT
    from fsctep_b200 import systems
    from fsctep_b200.ictd import ICTDConfig, ICTDEngine
    from fsctep_b200.models import reference_state_dict_shapes
    from fsctep_b200.neighbors import build_graph
    from fsctep_b200.weights import seeded_state_dict

    cfg = ICTDConfig(channels=channels, num_interaction=3, number_of_basis=8, max_radius=5.0,
                     function_type="gaussian", max_atomvalue=16)
    eng = ICTDEngine(seeded_state_dict(reference_state_dict_shapes(cfg), 13), cfg, "cuda")
    if kind == "diamond":
        s = systems.diamond_crystal(n_cells=(4, 4, 3), seed=29)
    else:
        s = systems.random_frames(n_frames=3, n_atoms=96, box=9.0, seed=30)
    dev = torch.device("cuda")
    pos, cell = torch.tensor(s["pos"], device=dev), torch.tensor(s["cell"], device=dev)
    b_np = s["batch"]
    fp = np.concatenate([[0], np.cumsum(np.bincount(b_np, minlength=s["cell"].shape[0]))])
    g = build_graph(pos, cell, 5.0, frame_ptr=fp)
    deg = (g.row_ptr[1:] - g.row_ptr[:-1]).cpu().numpy()
    assert deg.min() > 0 and (kind == "diamond" or (deg % 14 != 0).any())
    Z, b = torch.tensor(s["Z"], device=dev), torch.tensor(b_np, device=dev)
    try:
        ref = eng.energy_forces(pos, Z, b, cell, g)
        torch.cuda.synchronize()
        NAT.lib().fsc_ictd_set_conv2_path(1)
        out = eng.energy_forces(pos, Z, b, cell, g)
        again = eng.energy_forces(pos, Z, b, cell, g)
        torch.cuda.synchronize()
        assert eng.status() == 0
    finally:
        NAT.lib().fsc_ictd_set_conv2_path(0)
    assert torch.equal(out["energy"], ref["energy"])
    assert U.rel_max(out["forces"].cpu().numpy(), ref["forces"].cpu().numpy()) <= 2e-5
    assert U.rel_max(out["stress"].cpu().numpy(), ref["stress"].cpu().numpy()) <= 2e-5
    assert torch.equal(out["forces"], again["forces"]) and torch.equal(out["virial"], again["virial"])
