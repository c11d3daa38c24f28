"""The drop-in modules called the way the reference's LAMMPS ML-IAP wrapper calls them.

``interfaces/lammps_mliap.py:745-760`` (AtomForcesWrapper) passes zero positions that require
grad, ``edge_vec = pos[dst] - pos[src] + rij`` as ``precomputed_edge_vec`` and differentiates the
energy w.r.t. ``pos``; the traced core (``_TorchScriptEdgeVecCore``, ``:372-420``) takes edge_vec
as a positional input, and the legacy wrapper differentiates w.r.t. edge_vec itself.  Energies
and forces must match the reference's fp64 outputs on the golden fixtures.

The pure-cartesian-sparse reference accepts ``precomputed_edge_vec`` but never reads it (its
forward always rebuilds edge vectors from pos, shifts and cell), so there the drop-in gives
the result of the positions, like the reference.
"""

import numpy as np
import pytest
import torch

import golden_io
import gpu_util as U
from fsctep_b200.models import PureCartesianICTDTransformerLayer

pytestmark = [pytest.mark.gpu, U.needs_gpu]


def _ictd_module(cfg):
    return PureCartesianICTDTransformerLayer(max_embed_radius=float(cfg["max_radius"]), main_max_radius=5.0,
                                             main_number_of_basis=int(cfg["number_of_basis"]),
                                             hidden_dim_conv=int(cfg["channels"]),
                                             num_interaction=int(cfg["num_interaction"]),
                                             function_type_main=str(cfg["function_type"]),
                                             max_atomvalue=int(cfg["max_atomvalue"]))


def _case(kind, tag):
    if kind == "ictd":
        cfg, sd, c = golden_io.model_case(tag)
        m = _ictd_module(cfg)
    elif kind == "o3":
        from test_models_cpu import _o3_module

        cfg, sd, c = golden_io.o3_case(tag)
        m = _o3_module(cfg, device="cpu")
    else:
        from test_models_cpu import _sparse_module

        cfg, sd, c = golden_io.sparse_case(tag)
        m = _sparse_module(cfg, device="cpu")
    m.load_state_dict({k: v.float() for k, v in sd.items()})
    return m.cuda(), c


def _rij(c, dev):
    """Edge vectors in fp64, rounded once to fp32 (what LAMMPS hands over)."""
    pos, cell = torch.tensor(c["pos"]), torch.tensor(c["cell"])
    src, dst = torch.tensor(c["edge_src"]).long(), torch.tensor(c["edge_dst"]).long()
    sh = torch.tensor(c["edge_shifts"]).double()
    b = torch.tensor(c["batch"]).long()
    r = pos[dst] - pos[src] + torch.einsum("ni,nij->nj", sh, cell.double()[b[src]])
    return r.float().to(dev)


def _call(m, kind, c, pos, edge_vec, dev):
    kw = {"precomputed_edge_vec": edge_vec}
    if kind == "o3":
        kw["external_tensor"] = torch.tensor(c["field"], device=dev)
    args = (pos, torch.tensor(c["Z"], device=dev), torch.tensor(c["batch"], device=dev),
            torch.tensor(c["edge_src"], device=dev), torch.tensor(c["edge_dst"], device=dev),
            torch.tensor(c["edge_shifts"], device=dev).float(), torch.tensor(c["cell"], device=dev).float())
    return m(*args, **kw)


def _graph_energy(e, c, dev):
    b = torch.tensor(c["batch"], device=dev)
    B = c["cell"].shape[0]
    return torch.zeros(B, device=dev, dtype=e.dtype).index_add(0, b, e.view(-1))


@pytest.mark.parametrize("kind,tag", [("ictd", "a"), ("ictd", "c"), ("o3", "a"), ("o3", "b")])
def test_atom_forces_wrapper_pattern(kind, tag):
    """Zero positions + edge_vec = pos[dst] - pos[src] + rij; forces = -dE/dpos."""
    m, c = _case(kind, tag)
    dev = torch.device("cuda")
    rij = _rij(c, dev)
    n = c["pos"].shape[0]
    pos = torch.zeros(n, 3, device=dev, requires_grad=True)
    src, dst = torch.tensor(c["edge_src"], device=dev).long(), torch.tensor(c["edge_dst"], device=dev).long()
    edge_vec = pos[dst] - pos[src] + rij
    e = _call(m, kind, c, pos, edge_vec, dev)
    Eg = _graph_energy(e, c, dev)
    (gp,) = torch.autograd.grad(Eg.sum(), [pos])
    E = Eg.detach().double().cpu().numpy()
    ref = c["ref64_energy"]
    assert np.all(np.abs(E - ref) <= U.E_RTOL * np.abs(ref).max()), (E, ref)
    assert U.rel_max(-gp.cpu().numpy(), c["ref64_forces"]) <= U.F_RTOL


@pytest.mark.parametrize("kind,tag", [("ictd", "b"), ("o3", "a")])
def test_traced_core_pattern_edge_vec_grad(kind, tag):
    """edge_vec as a leaf that requires grad (the traced core's positional input): dE/d(edge_vec)
    summed onto the atoms (+ to dst, - to src) is -F; the real positions play no part."""
    m, c = _case(kind, tag)
    dev = torch.device("cuda")
    edge_vec = _rij(c, dev).requires_grad_(True)
    pos = torch.tensor(c["pos"], device=dev, dtype=torch.float32) + 17.0  # ignored with edge_vec given
    e = _call(m, kind, c, pos, edge_vec, dev)
    Eg = _graph_energy(e, c, dev)
    (ge,) = torch.autograd.grad(Eg.sum(), [edge_vec])
    n = c["pos"].shape[0]
    src, dst = torch.tensor(c["edge_src"], device=dev).long(), torch.tensor(c["edge_dst"], device=dev).long()
    dEdpos = torch.zeros(n, 3, device=dev).index_add(0, dst, ge).index_add(0, src, -ge)
    E = Eg.detach().double().cpu().numpy()
    ref = c["ref64_energy"]
    assert np.all(np.abs(E - ref) <= U.E_RTOL * np.abs(ref).max()), (E, ref)
    assert U.rel_max(-dEdpos.cpu().numpy(), c["ref64_forces"]) <= U.F_RTOL


def test_edge_vec_matches_position_path():
    """Same energies as the position path, with the edge order shuffled; finite edge gradients."""
    m, c = _case("ictd", "a")
    dev = torch.device("cuda")
    E = c["edge_src"].shape[0]
    perm = torch.randperm(E, generator=torch.Generator().manual_seed(3)).to(dev)
    rij = _rij(c, dev)[perm].requires_grad_(True)
    cc = dict(c)
    for k in ("edge_src", "edge_dst", "edge_shifts"):
        cc[k] = c[k][perm.cpu().numpy()]
    e1 = _call(m, "ictd", cc, torch.zeros(c["pos"].shape[0], 3, device=dev), rij, dev)
    pos = torch.tensor(c["pos"], device=dev, dtype=torch.float32)
    args = (pos, torch.tensor(c["Z"], device=dev), torch.tensor(c["batch"], device=dev),
            torch.tensor(c["edge_src"], device=dev), torch.tensor(c["edge_dst"], device=dev),
            torch.tensor(c["edge_shifts"], device=dev).float(), torch.tensor(c["cell"], device=dev).float())
    e0 = m(*args)
    assert (e1 - e0).abs().max().item() <= 1e-5 * e0.abs().max().item()
    (g,) = torch.autograd.grad(e1.sum(), [rij])
    assert torch.isfinite(g).all() and g.abs().max().item() > 0


@pytest.mark.parametrize("tag", ["a", "c"])
def test_sparse_ignores_edge_vec_like_the_reference(tag):
    m, c = _case("sparse", tag)
    dev = torch.device("cuda")
    pos = torch.tensor(c["pos"], device=dev, dtype=torch.float32).requires_grad_(True)
    junk = torch.zeros(c["edge_src"].shape[0], 3, device=dev)
    e = _call(m, "sparse", c, pos, junk, dev)
    (g,) = torch.autograd.grad(e.sum(), [pos])
    E = e.sum().item()
    assert abs(E - c["ref64_energy"].sum()) <= U.E_RTOL * abs(c["ref64_energy"].sum())
    assert U.rel_max(-g.cpu().numpy(), c["ref64_forces"]) <= U.F_RTOL
