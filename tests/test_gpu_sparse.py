"""GPU parity of the native pure-cartesian-sparse path against the reference's own outputs."""

import numpy as np
import pytest
import torch

import golden_io
import gpu_util as U
from fsctep_b200.ictd import GraphCSR
from fsctep_b200.sparse import SparseConfig, SparseEngine

pytestmark = [pytest.mark.gpu, U.needs_gpu]


def sparse_engine(tag):
    cfg, sd, c = golden_io.sparse_case(tag)
    scfg = SparseConfig(channels=int(cfg["channels"]), lmax=int(cfg["lmax"]),
                        num_interaction=int(cfg["num_interaction"]), number_of_basis=int(cfg["number_of_basis"]),
                        max_radius=float(cfg["max_radius"]), function_type=str(cfg["function_type"]),
                        max_atomvalue=int(cfg["max_atomvalue"]))
    eng = SparseEngine(sd, scfg, "cuda")
    dev = torch.device("cuda")
    g = GraphCSR.from_edges(torch.tensor(c["edge_src"], device=dev).long(), torch.tensor(c["edge_dst"], device=dev).long(),
                            torch.tensor(c["edge_shifts"], device=dev).float(), int(c["pos"].shape[0]))
    inputs = (torch.tensor(c["pos"], device=dev), torch.tensor(c["Z"], device=dev), torch.tensor(c["batch"], device=dev),
              torch.tensor(c["cell"], device=dev))
    return eng, g, inputs, c


@pytest.mark.parametrize("tag", ["a", "b", "e", "z"])
def test_sparse_energy_forces_stress_match_reference(tag):
    eng, g, (pos, Z, batch, cell), c = sparse_engine(tag)
    out = eng.energy_forces(pos, Z, batch, cell, g)
    torch.cuda.synchronize()
    assert eng.status() == 0
    E = out["energy"].double().cpu().numpy()
    assert np.all(np.abs(E - c["ref64_energy"]) <= U.E_RTOL * np.abs(c["ref64_energy"])), (E, c["ref64_energy"])
    assert U.rel_max(out["forces"].cpu().numpy(), c["ref64_forces"]) <= U.F_RTOL, \
        U.rel_max(out["forces"].cpu().numpy(), c["ref64_forces"])
    assert U.rel_max(out["stress"].cpu().numpy(), c["ref64_stress"]) <= U.S_RTOL
    np.testing.assert_allclose(out["atom_energy"].cpu().numpy(), c["ref64_atom_energy"], rtol=1e-4, atol=1e-4)


@pytest.mark.parametrize("gemm_path", [0, 1])
@pytest.mark.parametrize("tag", ["a", "d"])
def test_sparse_forces_sum_to_zero_and_repeat_bit_for_bit(tag, gemm_path):
    """The reverse pass has no floating-point atomics (dm rows reduced in a fixed order through the
    transpose CSR): energies, forces and the virial repeat bit for bit."""
    from fsctep_b200 import _native as NAT

    eng, g, (pos, Z, batch, cell), c = sparse_engine(tag)
    NAT.lib().fsc_ictd_set_gemm_path(gemm_path)
    try:
        outs = []
        for _ in range(3):
            o = eng.energy_forces(pos, Z, batch, cell, g)
            outs.append({k: o[k].clone() for k in ("energy", "forces", "virial")})
        torch.cuda.synchronize()
    finally:
        NAT.lib().fsc_ictd_set_gemm_path(0)
    F = outs[0]["forces"].double()
    assert F.sum(0).abs().max().item() < 1e-3 * F.abs().max().item()
    for o in outs[1:]:
        for k in ("energy", "forces", "virial"):
            assert torch.equal(outs[0][k], o[k]), k


def _dense_case(n_atoms=64, box=6.0, seed=11):
    """A dense periodic box (about 100-150 neighbours per atom within 5 A), so that nodes span the
    tensor-core kernels' 64-edge chunks and 128-edge groups; species drawn from the fixture's."""
    rng = np.random.default_rng(seed)
    pos = []
    while len(pos) < n_atoms:
        p = rng.uniform(0.0, box, 3)
        if all(np.linalg.norm((p - q + box / 2) % box - box / 2) >= 0.9 for q in pos):
            pos.append(p)
    pos = np.asarray(pos)
    Z = rng.choice([1, 8], size=n_atoms)
    return pos, Z, (np.eye(3) * box)[None]


@pytest.mark.parametrize("gemm_path", [0, 1])
def test_sparse_dense_graph_matches_oracle(gemm_path):
    """Tensor-core (path 0) and CUDA-core (path 1) aggregation kernels against the fp64 oracle on
    receivers with more than 64 and more than 128 incoming edges."""
    from fsctep_b200 import _native as NAT
    from oracle import neighbors as ON
    from oracle import sparse_model as SP
    from oracle.ictd_model import ICTDConfig as OCfg

    cfg, sd, _ = golden_io.sparse_case("a")
    pos, Z, cell = _dense_case()
    src, dst, S = ON.neighbor_list(pos, cell[0], float(cfg["max_radius"]))
    deg = np.bincount(dst, minlength=len(pos))
    assert deg.max() > 128 and deg.min() > 64, (deg.min(), deg.max())
    ocfg = OCfg(channels=int(cfg["channels"]), lmax=int(cfg["lmax"]), num_interaction=int(cfg["num_interaction"]),
                number_of_basis=int(cfg["number_of_basis"]), function_type=str(cfg["function_type"]),
                max_atomvalue=int(cfg["max_atomvalue"]))
    batch = np.zeros(len(pos), dtype=np.int64)
    ref = SP.sparse_energy_forces_stress(sd, ocfg, torch.tensor(pos), torch.tensor(Z), torch.tensor(batch),
                                         torch.tensor(src), torch.tensor(dst), torch.tensor(S, dtype=torch.float64),
                                         torch.tensor(cell))
    scfg = SparseConfig(channels=int(cfg["channels"]), lmax=int(cfg["lmax"]),
                        num_interaction=int(cfg["num_interaction"]), number_of_basis=int(cfg["number_of_basis"]),
                        max_radius=float(cfg["max_radius"]), function_type=str(cfg["function_type"]),
                        max_atomvalue=int(cfg["max_atomvalue"]))
    dev = torch.device("cuda")
    g = GraphCSR.from_edges(torch.tensor(src, device=dev), torch.tensor(dst, device=dev),
                            torch.tensor(S, device=dev).float(), len(pos))
    NAT.lib().fsc_ictd_set_gemm_path(gemm_path)
    try:
        eng = SparseEngine(sd, scfg, "cuda")
        out = eng.energy_forces(torch.tensor(pos, device=dev), torch.tensor(Z, device=dev),
                                torch.tensor(batch, device=dev), torch.tensor(cell, device=dev), g)
        torch.cuda.synchronize()
        assert eng.status() == 0
    finally:
        NAT.lib().fsc_ictd_set_gemm_path(0)
    E, E_ref = out["energy"].double().cpu().numpy(), ref["energy"].numpy()
    assert np.all(np.abs(E - E_ref) <= U.E_RTOL * np.abs(E_ref)), (E, E_ref)
    assert U.rel_max(out["forces"].cpu().numpy(), ref["forces"].numpy()) <= U.F_RTOL
    assert U.rel_max(out["stress"].cpu().numpy(), ref["stress"].numpy()) <= U.S_RTOL
