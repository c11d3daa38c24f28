"""Spatial decomposition with the native engine on one GPU: all ranks of a 2x1x1 and a 2x2x2
decomposition run in one process (run_local) and must reproduce the single-domain energy,
forces and virial."""

import numpy as np
import pytest
import torch

import gpu_util as U
from fsctep_b200 import _native as NAT
from fsctep_b200 import domain as D
from fsctep_b200 import systems
from fsctep_b200.ictd import ICTDConfig, ICTDEngine
from fsctep_b200.models import reference_state_dict_shapes
from fsctep_b200.neighbors import build_graph
from fsctep_b200.weights import seeded_state_dict

pytestmark = [pytest.mark.gpu, U.needs_gpu]


def _owned(dec, rank, pos, cell):
    frac = pos @ np.linalg.inv(cell)
    frac = frac - np.floor(frac)
    b = dec.block_of(rank)
    m = np.ones(len(frac), dtype=bool)
    for k in range(3):
        m &= np.floor(frac[:, k] * dec.dims[k]).astype(int) == b[k]
    return np.nonzero(m)[0]


@pytest.mark.parametrize("restrict", [False, True])
@pytest.mark.parametrize("dims", [(2, 1, 1), (2, 2, 2)])
def test_decomposed_engine_matches_single_domain(dims, restrict):
    """``restrict``: the engine evaluates layer k only within nint - 1 - k shells of the owned
    atoms (graph layer_atoms); the result must not change."""
    cfg = ICTDConfig(channels=32, num_interaction=3, number_of_basis=8, max_radius=5.0, function_type="gaussian",
                     max_atomvalue=16)
    eng = ICTDEngine(seeded_state_dict(reference_state_dict_shapes(cfg), 7), cfg, "cuda")
    s = systems.diamond_crystal(n_cells=(6, 6, 6), seed=41)
    dev = torch.device("cuda")
    pos, cell = torch.tensor(s["pos"], device=dev), torch.tensor(s["cell"], device=dev)
    Z = torch.tensor(s["Z"], device=dev, dtype=torch.int32)
    g = build_graph(pos, cell, 5.0)
    ref = eng.energy_forces(pos, Z, torch.zeros_like(Z), cell, g)
    ref_e = ref["energy"].double().item()
    ref_f = ref["forces"].double().cpu().numpy()
    ref_v = ref["virial"][0].double().cpu().numpy()

    c0 = s["cell"][0]
    dec = D.Decomposition(c0, dims, cfg.num_interaction * cfg.max_radius)
    ev0 = D.ictd_evaluator(eng, c0, cfg.max_radius, want_virial=True, restrict_layers=restrict)

    def ev(*a):
        out = ev0(*a)
        assert eng.status() == 0  # no receiver read a sender outside the previous layer's atoms
        return out

    owned = [_owned(dec, r, s["pos"], c0) for r in range(dec.world)]
    gens = [D.decomposed_step(dec, r, pos[torch.tensor(o, device=dev)], Z[torch.tensor(o, device=dev)], ev,
                              want_virial=True) for r, o in enumerate(owned)]
    res = D.run_local(gens)
    torch.cuda.synchronize()
    assert eng.status() == 0
    F = np.zeros_like(ref_f)
    for o, r in zip(owned, res):
        F[o] = r["forces"].double().cpu().numpy()
        assert abs(r["energy"].item() - ref_e) <= 1e-5 * abs(ref_e), (r["energy"].item(), ref_e)
        assert U.rel_max(r["virial"].cpu().numpy(), ref_v) <= 1e-4
    assert U.rel_max(F, ref_f) <= 1e-4, U.rel_max(F, ref_f)
    assert all(r["num_ghosts"] > 0 for r in res)


@pytest.mark.parametrize("dims", [(2, 1, 1), (2, 2, 2)])
def test_layer_exchange_matches_single_domain(dims):
    """Per-layer ghost-feature exchange (one-cutoff halo, the engine run in steps, ghost rows
    overwritten from their owners after every layer and their gradients returned) reproduces the
    single-domain energy, forces and virial."""
    cfg = ICTDConfig(channels=32, num_interaction=3, number_of_basis=8, max_radius=5.0, function_type="gaussian",
                     max_atomvalue=16)
    eng = ICTDEngine(seeded_state_dict(reference_state_dict_shapes(cfg), 7), cfg, "cuda")
    s = systems.diamond_crystal(n_cells=(6, 6, 6), seed=41)
    dev = torch.device("cuda")
    pos, cell = torch.tensor(s["pos"], device=dev), torch.tensor(s["cell"], device=dev)
    Z = torch.tensor(s["Z"], device=dev, dtype=torch.int32)
    g = build_graph(pos, cell, 5.0)
    ref = eng.energy_forces(pos, Z, torch.zeros_like(Z), cell, g)
    ref_e = ref["energy"].double().item()
    ref_f = ref["forces"].double().cpu().numpy()
    ref_v = ref["virial"][0].double().cpu().numpy()
    c0 = s["cell"][0]
    dec = D.Decomposition(c0, dims, cfg.max_radius)
    owned = [_owned(dec, r, s["pos"], c0) for r in range(dec.world)]
    F = np.zeros_like(ref_f)
    for r, o in enumerate(owned):
        # one engine per emulated rank: each keeps its own workspace across the interleaved steps
        er = ICTDEngine(seeded_state_dict(reference_state_dict_shapes(cfg), 7), cfg, "cuda")
        owned[r] = (o, er)
    gens = [D.layer_exchange_step(dec, r, pos[torch.tensor(o, device=dev)], Z[torch.tensor(o, device=dev)], er,
                                  cfg.max_radius, want_virial=True) for r, (o, er) in enumerate(owned)]
    res = D.run_local(gens)
    torch.cuda.synchronize()
    for (o, er), r in zip(owned, res):
        assert er.status() == 0
        F[o] = r["forces"].double().cpu().numpy()
        assert abs(r["energy"].item() - ref_e) <= 1e-5 * abs(ref_e), (r["energy"].item(), ref_e)
        assert U.rel_max(r["virial"].cpu().numpy(), ref_v) <= 1e-4
        assert r["num_ghosts"] > 0
    assert U.rel_max(F, ref_f) <= 1e-4, U.rel_max(F, ref_f)


def test_layer_atoms_contract_violation_is_reported():
    """A layer_atoms that cuts through the receptive field (layer 1 evaluated on atoms whose
    senders layer 0 skipped) is reported as status 70, not read from stale memory."""
    cfg = ICTDConfig(channels=32, num_interaction=3, number_of_basis=8, max_radius=5.0, function_type="gaussian",
                     max_atomvalue=16)
    eng = ICTDEngine(seeded_state_dict(reference_state_dict_shapes(cfg), 7), cfg, "cuda")
    s = systems.diamond_crystal(n_cells=(4, 4, 4), seed=5)
    dev = torch.device("cuda")
    pos, cell = torch.tensor(s["pos"], device=dev), torch.tensor(s["cell"], device=dev)
    Z = torch.tensor(s["Z"], device=dev, dtype=torch.int32)
    g = build_graph(pos, cell, 5.0)
    n = int(pos.shape[0])
    eng.forward(pos, Z, torch.zeros_like(Z), cell, g, num_local=8, layer_atoms=[n, n, n])
    assert eng.status() == 0
    eng.forward(pos, Z, torch.zeros_like(Z), cell, g, num_local=8, layer_atoms=[16, 16, 8])
    assert eng.status() == 70
    with pytest.raises(NAT.NativeError):
        eng.forward(pos, Z, torch.zeros_like(Z), cell, g, num_local=8, layer_atoms=[16, 32, 8])  # increasing


@pytest.mark.parametrize("dims", [(2, 1, 1), (2, 2, 1)])
def test_decomposed_sparse_engine_matches_single_domain(dims):
    """The pure-cartesian-sparse engine behind the same decomposition (halo = 3 x cutoff)."""
    from fsctep_b200.sparse import SparseConfig, SparseEngine
    import golden_io

    cfg, sd, _ = golden_io.sparse_case("b")  # lmax 3, FCC fixture weights
    scfg = SparseConfig(channels=int(cfg["channels"]), lmax=int(cfg["lmax"]),
                        num_interaction=int(cfg["num_interaction"]), number_of_basis=int(cfg["number_of_basis"]),
                        max_radius=float(cfg["max_radius"]), function_type=str(cfg["function_type"]),
                        max_atomvalue=int(cfg["max_atomvalue"]))
    eng = SparseEngine(sd, scfg, "cuda")
    s = systems.fcc_crystal(n_cells=(9, 9, 9), seed=43)
    dev = torch.device("cuda")
    pos, cell = torch.tensor(s["pos"], device=dev), torch.tensor(s["cell"], device=dev)
    Z = torch.tensor(s["Z"], device=dev, dtype=torch.int32)
    g = build_graph(pos, cell, 5.0)
    ref = eng.energy_forces(pos, Z, torch.zeros_like(Z), cell, g)
    ref_e = ref["energy"].double().item()
    ref_f = ref["forces"].double().cpu().numpy()
    ref_v = ref["virial"][0].double().cpu().numpy()

    c0 = s["cell"][0]
    dec = D.Decomposition(c0, dims, scfg.num_interaction * scfg.max_radius)
    ev = D.sparse_evaluator(eng, c0, scfg.max_radius, want_virial=True)
    owned = [_owned(dec, r, s["pos"], c0) for r in range(dec.world)]
    gens = [D.decomposed_step(dec, r, pos[torch.tensor(o, device=dev)], Z[torch.tensor(o, device=dev)], ev,
                              want_virial=True) for r, o in enumerate(owned)]
    res = D.run_local(gens)
    torch.cuda.synchronize()
    assert eng.status() == 0
    F = np.zeros_like(ref_f)
    for o, r in zip(owned, res):
        F[o] = r["forces"].double().cpu().numpy()
        assert abs(r["energy"].item() - ref_e) <= 1e-5 * abs(ref_e), (r["energy"].item(), ref_e)
        assert U.rel_max(r["virial"].cpu().numpy(), ref_v) <= 1e-4
    assert U.rel_max(F, ref_f) <= 1e-4, U.rel_max(F, ref_f)
    assert all(r["num_ghosts"] > 0 for r in res)


@pytest.mark.parametrize("dims", [(2, 1, 1), (2, 2, 1)])
def test_sparse_layer_exchange_matches_single_domain(dims):
    """The pure-cartesian-sparse engine with the per-layer ghost-feature exchange (one-cutoff halo,
    whole-system E / N through the owned edge and atom counts)."""
    from fsctep_b200.sparse import SparseConfig, SparseEngine
    import golden_io

    cfg, sd, _ = golden_io.sparse_case("b")
    scfg = SparseConfig(channels=int(cfg["channels"]), lmax=int(cfg["lmax"]),
                        num_interaction=int(cfg["num_interaction"]), number_of_basis=int(cfg["number_of_basis"]),
                        max_radius=float(cfg["max_radius"]), function_type=str(cfg["function_type"]),
                        max_atomvalue=int(cfg["max_atomvalue"]))
    eng = SparseEngine(sd, scfg, "cuda")
    s = systems.fcc_crystal(n_cells=(9, 9, 9), seed=43)
    dev = torch.device("cuda")
    pos, cell = torch.tensor(s["pos"], device=dev), torch.tensor(s["cell"], device=dev)
    Z = torch.tensor(s["Z"], device=dev, dtype=torch.int32)
    ref = eng.energy_forces(pos, Z, torch.zeros_like(Z), cell, build_graph(pos, cell, 5.0))
    ref_e = ref["energy"].double().item()
    ref_f = ref["forces"].double().cpu().numpy()
    ref_v = ref["virial"][0].double().cpu().numpy()
    c0 = s["cell"][0]
    dec = D.Decomposition(c0, dims, scfg.max_radius)
    owned = [_owned(dec, r, s["pos"], c0) for r in range(dec.world)]
    engines = [SparseEngine(sd, scfg, "cuda") for _ in owned]  # one workspace per emulated rank
    gens = [D.layer_exchange_step(dec, r, pos[torch.tensor(o, device=dev)], Z[torch.tensor(o, device=dev)],
                                  engines[r], scfg.max_radius, want_virial=True) for r, o in enumerate(owned)]
    res = D.run_local(gens)
    torch.cuda.synchronize()
    F = np.zeros_like(ref_f)
    for o, r, er in zip(owned, res, engines):
        assert er.status() == 0
        F[o] = r["forces"].double().cpu().numpy()
        assert abs(r["energy"].item() - ref_e) <= 1e-5 * abs(ref_e), (r["energy"].item(), ref_e)
        assert U.rel_max(r["virial"].cpu().numpy(), ref_v) <= 1e-4
    assert U.rel_max(F, ref_f) <= 1e-4, U.rel_max(F, ref_f)
