"""Pin the CPU oracle against golden vectors recorded from the reference itself."""

import numpy as np
import pytest
import torch

import golden_io
from oracle import ictd_tables as T
from oracle import ictd_model as OM
from oracle import neighbors as ON


def test_tables_match_reference():
    z = golden_io.load("ictd_tables.npz")
    for L in range(5):
        np.testing.assert_allclose(T.harmonic_basis(L).numpy(), z[f"basis_{L}"], rtol=0, atol=1e-13)
        np.testing.assert_allclose(T.direction_projector(L).numpy(), z[f"dirproj_{L}"], rtol=0, atol=1e-12)
    for lmax in (2, 3):
        paths = T.tp_paths(lmax)
        assert [tuple(p) for p in z[f"L{lmax}_paths"].tolist()] == paths
        for (l1, l2, l3) in paths:
            np.testing.assert_allclose(T.normalized_cg(l1, l2, l3).numpy(), z[f"L{lmax}_cg_{l1}{l2}{l3}"],
                                       rtol=0, atol=1e-13)
        groups = T.tp_groups(paths)
        for g, U in zip(groups, T.group_U(paths, groups)):
            np.testing.assert_allclose(U.numpy(), z[f"L{lmax}_U_{g['l1']}{g['l2']}"], rtol=0, atol=1e-13)
        f = [T.normalized_cg(l, l, 0)[0, 0, 0].item() for l in range(lmax + 1)]
        np.testing.assert_allclose(f, z[f"L{lmax}_p5_factors"], rtol=0, atol=1e-14)
    n = torch.tensor(z["dir_n"])
    for l in range(5):
        np.testing.assert_allclose(T.direction_harmonics(n, l).numpy(), z[f"dir_Y_{l}"], rtol=0, atol=1e-12)


def test_high_lmax_basis_orthonormal():
    """B^T G B = I (reference test/test_high_lmax.py:21-37)."""
    for L in range(0, 8):
        B = T.harmonic_basis(L)
        G = T.gram_gaussian(L)
        np.testing.assert_allclose((B.T @ G @ B).numpy(), np.eye(2 * L + 1), atol=1e-10)


@pytest.mark.parametrize("tag", ["a", "b", "c", "e", "z"])
def test_oracle_energy_forces_stress_match_reference(tag):
    cfg, sd, c = golden_io.model_case(tag)
    ocfg = OM.ICTDConfig(**cfg)
    out = OM.energy_forces_stress(
        sd, ocfg, torch.tensor(c["pos"]), torch.tensor(c["Z"]), torch.tensor(c["batch"]),
        torch.tensor(c["edge_src"]).long(), torch.tensor(c["edge_dst"]).long(),
        torch.tensor(c["edge_shifts"]).double(), torch.tensor(c["cell"]))
    np.testing.assert_allclose(out["energy"].numpy(), c["ref64_energy"], rtol=1e-10, atol=1e-10)
    np.testing.assert_allclose(out["forces"].numpy(), c["ref64_forces"], rtol=1e-9, atol=1e-10)
    np.testing.assert_allclose(out["stress"].numpy(), c["ref64_stress"], rtol=1e-9, atol=1e-11)


@pytest.mark.parametrize("tag", ["a", "b", "c", "e", "z"])
def test_neighbor_oracle_reproduces_fixture(tag):
    _, _, c = golden_io.model_case(tag)
    src, dst, S = ON.batched_neighbor_list(c["pos"], c["batch"], c["cell"], 5.0, tuple(c["pbc"]))
    np.testing.assert_array_equal(src, c["edge_src"])
    np.testing.assert_array_equal(dst, c["edge_dst"])
    np.testing.assert_array_equal(S, c["edge_shifts"])
