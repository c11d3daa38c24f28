"""core.pt round trip on the GPU: export, torch.jit.load (and freeze), then the LAMMPS engine's
call sequence (edge_vec = pos[dst] - pos[src] + shift with autograd, grad of the local energy
with respect to pos and shift) against the native engine."""

import numpy as np
import pytest
import torch

import gpu_util as U
from fsctep_b200 import torchscript as TS

pytestmark = [pytest.mark.gpu, U.needs_gpu]


def _lammps_like(core, c, nlocal):
    dev = torch.device("cuda")
    pos = torch.tensor(c["pos"], device=dev, dtype=torch.float32).requires_grad_(True)
    A = torch.tensor(c["Z"], device=dev).long()
    batch = torch.zeros(pos.shape[0], dtype=torch.long, device=dev)
    src = torch.tensor(c["edge_src"], device=dev).long()
    dst = torch.tensor(c["edge_dst"], device=dev).long()
    shifts = torch.tensor(c["edge_shifts"], device=dev, dtype=torch.float32)
    cell = torch.tensor(c["cell"], device=dev, dtype=torch.float32)[:1]
    shift_vec = torch.einsum("ni,nij->nj", shifts, cell[batch[src]])
    shift_leaf = shift_vec.clone().detach().requires_grad_(True)
    edge_vec = pos[dst] - pos[src] + shift_leaf
    atom_e = core(pos, A, batch, src, dst, shifts, cell, edge_vec, torch.empty(0, device=dev))
    E_local = atom_e.view(-1)[:nlocal].sum()
    gpos, gshift = torch.autograd.grad(E_local, [pos, shift_leaf])
    virial = (edge_vec.detach().T @ gshift).cpu().numpy()
    return atom_e.detach().view(-1).cpu().numpy(), -gpos.cpu().numpy(), virial


@pytest.mark.parametrize("freeze", [False, True])
def test_core_pt_matches_engine(tmp_path, freeze):
    eng, g, (pos, Z, batch, cell), c, icfg, sd = U.golden_engine("a")
    # one frame: the LAMMPS engine evaluates one periodic cell
    n0 = int((c["batch"] == 0).sum())
    e_mask = c["batch"][c["edge_dst"]] == 0
    c1 = {"pos": c["pos"][:n0], "Z": c["Z"][:n0], "edge_src": c["edge_src"][e_mask],
          "edge_dst": c["edge_dst"][e_mask], "edge_shifts": c["edge_shifts"][e_mask], "cell": c["cell"][:1]}
    path = str(tmp_path / "core.pt")
    TS.export_core(sd, icfg, path)
    core = torch.jit.load(path, map_location="cuda")
    if freeze:
        core = torch.jit.freeze(core.eval())
    nlocal = n0 - 7
    ae, F, W = _lammps_like(core, c1, nlocal)

    from fsctep_b200.ictd import GraphCSR
    dev = torch.device("cuda")
    g1 = GraphCSR.from_edges(torch.tensor(c1["edge_src"], device=dev).long(),
                             torch.tensor(c1["edge_dst"], device=dev).long(),
                             torch.tensor(c1["edge_shifts"], device=dev).float(), n0)
    ref = eng.energy_forces(torch.tensor(c1["pos"], device=dev), torch.tensor(c1["Z"], device=dev),
                            torch.zeros(n0, dtype=torch.int32, device=dev), torch.tensor(c1["cell"], device=dev),
                            g1, num_local=nlocal)
    torch.cuda.synchronize()
    np.testing.assert_allclose(ae, ref["atom_energy"].cpu().numpy(), rtol=1e-5, atol=1e-6)
    assert U.rel_max(F, ref["forces"].cpu().numpy()) <= 1e-5
    assert U.rel_max(W, ref["virial"][0].cpu().numpy()) <= 1e-5
    # the custom op is the only compute in the graph
    assert "fsctep::ictd_atom_energy" in str(core.graph) or freeze


def test_double_backward_is_refused(tmp_path):
    eng, g, _, c, icfg, sd = U.golden_engine("a")
    core = TS.ICTDCore(sd, icfg).eval()
    dev = torch.device("cuda")
    args = TS._example_inputs("cuda", icfg.max_atomvalue)
    ev = args[7].clone().requires_grad_(True)
    e = core(*args[:7], ev, args[8]).sum()
    with pytest.raises(RuntimeError, match="double backward"):
        torch.autograd.grad(e, ev, create_graph=True)


def _one_graph(c, b=0):
    """Graph b of a batched fixture as a one-graph case (atoms renumbered from 0)."""
    idx = np.nonzero(c["batch"] == b)[0]
    n0 = idx[0]
    e = np.nonzero(c["batch"][c["edge_dst"]] == b)[0]
    return {"pos": c["pos"][idx], "Z": c["Z"][idx], "edge_src": c["edge_src"][e] - n0,
            "edge_dst": c["edge_dst"][e] - n0, "edge_shifts": c["edge_shifts"][e], "cell": c["cell"][b:b + 1]}


def _lammps_like_field(core, c, nlocal, field):
    dev = torch.device("cuda")
    pos = torch.tensor(c["pos"], device=dev, dtype=torch.float32).requires_grad_(True)
    A = torch.tensor(c["Z"], device=dev).long()
    batch = torch.zeros(pos.shape[0], dtype=torch.long, device=dev)
    src = torch.tensor(c["edge_src"], device=dev).long()
    dst = torch.tensor(c["edge_dst"], device=dev).long()
    shifts = torch.tensor(c["edge_shifts"], device=dev, dtype=torch.float32)
    cell = torch.tensor(c["cell"], device=dev, dtype=torch.float32)[:1]
    edge_vec = pos[dst] - pos[src] + torch.einsum("ni,nij->nj", shifts, cell[batch[src]])
    atom_e = core(pos, A, batch, src, dst, shifts, cell, edge_vec, field)
    (gpos,) = torch.autograd.grad(atom_e.view(-1)[:nlocal].sum(), [pos])
    return atom_e.detach().view(-1).cpu().numpy(), -gpos.cpu().numpy()


def test_o3_core_pt_with_field_matches_reference(tmp_path):
    """pure-cartesian-ictd-o3 core.pt with its external field as the traced core's external_tensor."""
    import golden_io
    from fsctep_b200.ictd import ICTDConfig

    cfg, sd, c = golden_io.o3_case("a")
    icfg = ICTDConfig(channels=int(cfg["channels"]), lmax=2, num_interaction=int(cfg["num_interaction"]),
                      number_of_basis=int(cfg["number_of_basis"]), max_radius=float(cfg["max_radius"]),
                      function_type=str(cfg["function_type"]), max_atomvalue=int(cfg["max_atomvalue"]), o3=True)
    path = str(tmp_path / "core_o3.pt")
    TS.export_core(sd, icfg, path)
    core = torch.jit.load(path, map_location="cuda")
    c1 = _one_graph(c, 0)
    field = torch.tensor(c["field"][0], device="cuda", dtype=torch.float32)
    n = c1["pos"].shape[0]
    ae, F = _lammps_like_field(core, c1, n, field)
    assert abs(ae.sum() - c["ref64_energy"][0]) <= U.E_RTOL * np.abs(c["ref64_energy"]).max()
    ref_f = c["ref64_forces"][c["batch"] == 0]
    assert U.rel_max(F, ref_f) <= U.F_RTOL
    np.testing.assert_allclose(ae, c["ref64_atom_energy"][c["batch"] == 0], rtol=1e-4, atol=1e-4)


def test_sparse_core_pt_matches_reference(tmp_path):
    import golden_io
    from fsctep_b200.sparse import SparseConfig

    cfg, sd, c = golden_io.sparse_case("a")
    scfg = SparseConfig(channels=int(cfg["channels"]), lmax=int(cfg["lmax"]),
                        num_interaction=int(cfg["num_interaction"]), number_of_basis=int(cfg["number_of_basis"]),
                        max_radius=float(cfg["max_radius"]), function_type=str(cfg["function_type"]),
                        max_atomvalue=int(cfg["max_atomvalue"]))
    path = str(tmp_path / "core_sparse.pt")
    TS.export_core(sd, scfg, path)
    core = torch.jit.freeze(torch.jit.load(path, map_location="cuda").eval())
    n = c["pos"].shape[0]
    ae, F, _ = _lammps_like(core, c, n)
    assert abs(ae.sum() - c["ref64_energy"].sum()) <= U.E_RTOL * abs(c["ref64_energy"].sum())
    assert U.rel_max(F, c["ref64_forces"]) <= U.F_RTOL
