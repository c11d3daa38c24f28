"""The drop-in module on the GPU: autograd forces and strain stress match the reference."""

import numpy as np
import pytest
import torch

import golden_io
import gpu_util as U
from fsctep_b200.models import PureCartesianICTDTransformerLayer

pytestmark = [pytest.mark.gpu, U.needs_gpu]


def test_autograd_forces_and_strain_stress():
    cfg, sd, c = golden_io.model_case("a")
    m = PureCartesianICTDTransformerLayer(max_embed_radius=5.0, main_max_radius=5.0, main_number_of_basis=8,
                                          hidden_dim_conv=32, num_interaction=2, function_type_main="bessel").cuda()
    m.load_state_dict({k: v.float() for k, v in sd.items()})
    dev = torch.device("cuda")
    pos = torch.tensor(c["pos"], device=dev, dtype=torch.float32, requires_grad=True)
    cell = torch.tensor(c["cell"], device=dev, dtype=torch.float32)
    batch = torch.tensor(c["batch"], device=dev)
    nb = cell.shape[0]
    strain = torch.zeros(nb, 3, 3, device=dev, requires_grad=True)
    D = torch.eye(3, device=dev) + 0.5 * (strain + strain.transpose(-1, -2))
    pos_in = torch.einsum("ni,nij->nj", pos, D[batch])
    cell_in = torch.bmm(cell, D)
    e = m(pos_in, torch.tensor(c["Z"], device=dev), batch, torch.tensor(c["edge_src"], device=dev).long(),
          torch.tensor(c["edge_dst"], device=dev).long(), torch.tensor(c["edge_shifts"], device=dev).float(), cell_in)
    assert e.shape == (pos.shape[0], 1)
    Eg = torch.zeros(nb, device=dev).index_add(0, batch, e.squeeze(-1))
    gp, gs = torch.autograd.grad(Eg.sum(), [pos, strain])
    vol = torch.abs(torch.det(cell.double())).float()
    stress = (gs / vol.view(-1, 1, 1)).cpu().numpy()
    assert np.all(np.abs(Eg.detach().cpu().numpy() - c["ref64_energy"]) <= U.E_RTOL * np.abs(c["ref64_energy"]))
    assert U.rel_max(-gp.cpu().numpy(), c["ref64_forces"]) <= U.F_RTOL
    assert U.rel_max(stress, c["ref64_stress"]) <= U.S_RTOL


def test_edge_order_does_not_matter():
    cfg, sd, c = golden_io.model_case("b")
    m = PureCartesianICTDTransformerLayer(max_embed_radius=5.0, main_max_radius=5.0, main_number_of_basis=8,
                                          hidden_dim_conv=int(cfg["channels"]), num_interaction=3,
                                          function_type_main="gaussian", max_atomvalue=16).cuda()
    m.load_state_dict({k: v.float() for k, v in sd.items()})
    dev = torch.device("cuda")
    E = c["edge_src"].shape[0]
    perm = torch.randperm(E, generator=torch.Generator().manual_seed(0))
    args = [torch.tensor(c["edge_src"]).long(), torch.tensor(c["edge_dst"]).long(),
            torch.tensor(c["edge_shifts"]).float()]
    pos = torch.tensor(c["pos"], device=dev, dtype=torch.float32)
    Z, b, cell = (torch.tensor(c[k], device=dev) for k in ("Z", "batch", "cell"))
    e1 = m(pos, Z, b, *[a.to(dev) for a in args], cell.float())
    e2 = m(pos, Z, b, *[a[perm].to(dev) for a in args], cell.float())
    torch.cuda.synchronize()
    assert (e1 - e2).abs().max().item() < 1e-5 * e1.abs().max().item()


@pytest.mark.parametrize("tag", ["a", "b"])
def test_o3_module_matches_reference(tag):
    """Drop-in o3 module with a reference checkpoint: energy, autograd forces and heads."""
    from test_models_cpu import _o3_module

    cfg, sd, c = golden_io.o3_case(tag)
    m = _o3_module(cfg, device="cpu")
    m.load_state_dict({k: v.float() for k, v in sd.items()})
    m = m.cuda()
    dev = torch.device("cuda")
    pos = torch.tensor(c["pos"], device=dev, dtype=torch.float32).requires_grad_(True)
    b = torch.tensor(c["batch"], device=dev)
    e, phys = m(pos, torch.tensor(c["Z"], device=dev), b, torch.tensor(c["edge_src"], device=dev),
                torch.tensor(c["edge_dst"], device=dev), torch.tensor(c["edge_shifts"], device=dev).float(),
                torch.tensor(c["cell"], device=dev).float(), external_tensor=torch.tensor(c["field"], device=dev),
                return_physical_tensors=True)
    B = c["cell"].shape[0]
    Eg = torch.zeros(B, device=dev, dtype=e.dtype).index_add(0, b, e.view(-1))
    (g,) = torch.autograd.grad(Eg.sum(), [pos])
    E = Eg.detach().double().cpu().numpy()
    assert np.all(np.abs(E - c["ref64_energy"]) <= U.E_RTOL * np.abs(c["ref64_energy"]).max())
    assert U.rel_max(-g.cpu().numpy(), c["ref64_forces"]) <= U.F_RTOL
    assert U.rel_max(phys["dipole"][1].cpu().numpy(), c["ref64_dipole"]) <= 1e-5
    assert U.rel_max(phys["polarizability"][2].cpu().numpy(), c["ref64_polar2"]) <= 1e-5


@pytest.mark.parametrize("tag", ["a", "b"])
def test_sparse_module_matches_reference(tag):
    from test_models_cpu import _sparse_module

    cfg, sd, c = golden_io.sparse_case(tag)
    m = _sparse_module(cfg, device="cpu")
    m.load_state_dict({k: v.float() for k, v in sd.items()})
    m = m.cuda()
    dev = torch.device("cuda")
    pos = torch.tensor(c["pos"], device=dev, dtype=torch.float32).requires_grad_(True)
    b = torch.tensor(c["batch"], device=dev)
    e = m(pos, torch.tensor(c["Z"], device=dev), b, torch.tensor(c["edge_src"], device=dev),
          torch.tensor(c["edge_dst"], device=dev), torch.tensor(c["edge_shifts"], device=dev).float(),
          torch.tensor(c["cell"], device=dev).float())
    (g,) = torch.autograd.grad(e.sum(), [pos])
    E = e.sum().item()
    assert abs(E - c["ref64_energy"].sum()) <= U.E_RTOL * abs(c["ref64_energy"].sum())
    assert U.rel_max(-g.cpu().numpy(), c["ref64_forces"]) <= U.F_RTOL
