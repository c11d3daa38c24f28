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
