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


@pytest.mark.parametrize("tag", ["a", "b"])
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


def test_sparse_forces_sum_to_zero_and_repeatable():
    eng, g, (pos, Z, batch, cell), c = sparse_engine("a")
    o1 = eng.energy_forces(pos, Z, batch, cell, g)
    e1 = o1["energy"].clone()
    o2 = eng.energy_forces(pos, Z, batch, cell, g)
    torch.cuda.synchronize()
    F = o1["forces"].double()
    assert F.sum(0).abs().max().item() < 1e-3 * F.abs().max().item()
    assert torch.equal(e1, o2["energy"])
