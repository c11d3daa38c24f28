"""GPU parity of the native pure-cartesian-ictd-o3 path (external 1o field, dipole and
polarizability heads) against the reference's own outputs."""

import numpy as np
import pytest
import torch

import golden_io
import gpu_util as U
from fsctep_b200.ictd import GraphCSR, ICTDConfig, ICTDEngine

pytestmark = [pytest.mark.gpu, U.needs_gpu]


def _engine(tag):
    cfg, sd, c = golden_io.o3_case(tag)
    icfg = ICTDConfig(channels=int(cfg["channels"]), lmax=int(cfg["lmax"]), num_interaction=int(cfg["num_interaction"]),
                      number_of_basis=int(cfg["number_of_basis"]), max_radius=float(cfg["max_radius"]),
                      function_type=str(cfg["function_type"]), max_atomvalue=int(cfg["max_atomvalue"]), o3=True)
    eng = ICTDEngine(sd, icfg, "cuda")
    dev = torch.device("cuda")
    g = GraphCSR.from_edges(torch.tensor(c["edge_src"], device=dev).long(), torch.tensor(c["edge_dst"], device=dev).long(),
                            torch.tensor(c["edge_shifts"], device=dev).float(), int(c["pos"].shape[0]))
    inputs = (torch.tensor(c["pos"], device=dev), torch.tensor(c["Z"], device=dev), torch.tensor(c["batch"], device=dev),
              torch.tensor(c["cell"], device=dev))
    return eng, g, inputs, c


@pytest.mark.parametrize("readout_path", [0, 1])
@pytest.mark.parametrize("tag", ["a", "b", "e"])
def test_o3_energy_forces_heads_match_reference(tag, readout_path):
    from fsctep_b200 import _native as NAT

    eng, g, (pos, Z, batch, cell), c = _engine(tag)
    try:
        NAT.lib().fsc_ictd_set_readout_path(readout_path)
        out = eng.energy_forces(pos, Z, batch, cell, g, want_stress=False, field=torch.tensor(c["field"]))
        heads = eng.heads()
        torch.cuda.synchronize()
        assert eng.status() == 0
    finally:
        NAT.lib().fsc_ictd_set_readout_path(0)
    E = out["energy"].double().cpu().numpy()
    ref_e = c["ref64_energy"]
    assert np.all(np.abs(E - ref_e) <= U.E_RTOL * np.abs(ref_e).max()), (E, ref_e)
    assert U.rel_max(out["forces"].cpu().numpy(), c["ref64_forces"]) <= U.F_RTOL
    np.testing.assert_allclose(out["atom_energy"].cpu().numpy(), c["ref64_atom_energy"], rtol=1e-4, atol=1e-4)
    assert U.rel_max(heads["dipole"][1].cpu().numpy(), c["ref64_dipole"]) <= 1e-5
    assert U.rel_max(heads["polarizability"][0].cpu().numpy(), c["ref64_polar0"]) <= 1e-5
    assert U.rel_max(heads["polarizability"][2].cpu().numpy(), c["ref64_polar2"]) <= 1e-5


def test_o3_field_changes_energy_and_is_linear_in_conv1():
    """Zero field differs from the drawn field; the field enters only conv1's l = 1 term."""
    eng, g, (pos, Z, batch, cell), c = _engine("a")
    e1 = eng.forward(pos, Z, batch, cell, g, field=torch.tensor(c["field"]))[0].clone()
    e0 = eng.forward(pos, Z, batch, cell, g, field=torch.zeros_like(torch.tensor(c["field"])))[0].clone()
    en = eng.forward(pos, Z, batch, cell, g)[0].clone()
    torch.cuda.synchronize()
    assert torch.equal(e0, en)
    assert (e1 - e0).abs().max().item() > 1e-6 * e0.abs().max().item()
