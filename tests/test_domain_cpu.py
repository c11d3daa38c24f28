"""Spatial decomposition host logic on CPU: halo exchange, ghost-force return, energy / virial
reduction.  A toy two-hop message-passing potential (receptive field 2 * rc, like a 2-layer
model) is evaluated on the whole periodic system and decomposed over 2, 4 and 8 ranks, in one
process (run_local) and over real gloo ranks (run_dist)."""

import socket

import numpy as np
import pytest
import torch

from fsctep_b200 import domain as D
from fsctep_b200 import systems
from oracle import neighbors as ON

RC = 4.0  # first two diamond shells (2.35 and 3.84 A)
NHOP = 2


def toy_evaluate(cell, restrict=False):
    """Evaluator of a 2-hop potential on a local system (owned atoms first).

    ``restrict`` evaluates it the way the engine does with ``layer_atoms``: ghosts reordered by
    distance shell (:func:`domain.layer_shells`), hop k only for receivers below
    ``layer_atoms[k]``, atom energies only below ``layer_atoms[-1]``; the contract that every
    evaluated receiver reads only senders evaluated one hop earlier is asserted."""
    cell_t = torch.tensor(cell, dtype=torch.float64)

    def evaluate(pos, species, num_local, pbc):
        n_all = pos.shape[0]
        perm = None
        if restrict:
            perm, L = D.layer_shells(pos, num_local, [not q for q in pbc], RC, NHOP)
            pos, species = pos[perm], species[perm]
        src, dst, S = ON.neighbor_list(pos.detach().numpy(), cell, RC, pbc=pbc)
        p = pos.detach().clone().requires_grad_(True)
        src_t, dst_t = torch.tensor(src), torch.tensor(dst)
        r = p[dst_t] - p[src_t] + torch.tensor(S, dtype=torch.float64) @ cell_t
        r.retain_grad()
        d = r.norm(dim=1)
        phi = (1.0 - d / RC) ** 2
        w = 1.0 + 0.1 * species.to(torch.float64)
        n = p.shape[0]
        m1 = torch.zeros(n, dtype=torch.float64).index_add(0, dst_t, phi * w[src_t])
        if restrict:
            assert bool((src_t[dst_t < L[1]] < L[0]).all())  # hop-2 receivers read hop-1 senders only
            m1 = torch.zeros(n, dtype=torch.float64).index_add(
                0, dst_t[dst_t < L[0]], (phi * w[src_t])[dst_t < L[0]])
            on2 = dst_t < L[1]
            m2 = torch.zeros(n, dtype=torch.float64).index_add(
                0, dst_t[on2], (phi * torch.tanh(0.3 * m1[src_t]))[on2])
        else:
            m2 = torch.zeros(n, dtype=torch.float64).index_add(0, dst_t, phi * torch.tanh(0.3 * m1[src_t]))
        e = 0.01 * m2 ** 2 + 0.5 * m1 + 0.05 * m1 * m2
        if restrict:
            e = torch.where(torch.arange(n) < L[-1], e, torch.zeros_like(e))
        E = e[:num_local].sum()
        E.backward()
        forces, ae = -p.grad, e.detach()
        if restrict:
            forces = torch.zeros(n_all, 3, dtype=torch.float64).index_copy(0, perm, forces)
            ae = torch.zeros(n_all, dtype=torch.float64).index_copy(0, perm, ae)
        return {"energy": E.detach(), "forces": forces, "atom_energy": ae, "virial": (r.detach().T @ r.grad)}

    return evaluate


def _system():
    s = systems.diamond_crystal(n_cells=(4, 4, 4), seed=31)
    s["Z"] = (np.arange(s["pos"].shape[0]) % 3).astype(np.int64)
    return s


def _reference(s):
    ev = toy_evaluate(s["cell"][0])
    pos = torch.tensor(s["pos"], dtype=torch.float64)
    return ev(pos, torch.tensor(s["Z"]), pos.shape[0], (True, True, True))


def _owned(dec, rank, s):
    frac = s["pos"] @ np.linalg.inv(s["cell"][0])
    frac = frac - np.floor(frac)
    b = dec.block_of(rank)
    m = np.ones(len(frac), dtype=bool)
    for k in range(3):
        m &= (np.floor(frac[:, k] * dec.dims[k]).astype(int) == b[k])
    return np.nonzero(m)[0]


def _decomposed_local(s, dims, halo, restrict=False):
    dec = D.Decomposition(s["cell"][0], dims, halo)
    ev = toy_evaluate(s["cell"][0], restrict)
    owned = [_owned(dec, r, s) for r in range(dec.world)]
    gens = [D.decomposed_step(dec, r, torch.tensor(s["pos"][o], dtype=torch.float64), torch.tensor(s["Z"][o]), ev,
                              want_virial=True) for r, o in enumerate(owned)]
    res = D.run_local(gens)
    F = np.zeros_like(s["pos"])
    for o, r in zip(owned, res):
        F[o] = r["forces"].numpy()
    return res, F, owned


@pytest.mark.parametrize("restrict", [False, True])
@pytest.mark.parametrize("dims", [(2, 1, 1), (2, 2, 1), (2, 2, 2), (1, 2, 1)])
def test_decomposed_matches_single_domain(dims, restrict):
    s = _system()
    ref = _reference(s)
    res, F, owned = _decomposed_local(s, dims, NHOP * RC, restrict)
    assert sorted(np.concatenate(owned).tolist()) == list(range(s["pos"].shape[0]))
    for r in res:
        assert abs(r["energy"].item() - ref["energy"].item()) <= 1e-10 * abs(ref["energy"].item())
        np.testing.assert_allclose(r["virial"].numpy(), ref["virial"].numpy(), rtol=1e-9, atol=1e-9)
    np.testing.assert_allclose(F, ref["forces"].numpy(), rtol=1e-9, atol=1e-10)
    ae = np.zeros(s["pos"].shape[0])
    for o, r in zip(owned, res):
        ae[o] = r["atom_energy"].numpy()
    np.testing.assert_allclose(ae, ref["atom_energy"].numpy(), rtol=1e-10, atol=1e-12)
    assert all(r["num_ghosts"] > 0 for r in res)


def test_short_halo_is_detected():
    """A halo shorter than the receptive field changes the energy: the test above has teeth."""
    s = _system()
    ref = _reference(s)
    res, _, _ = _decomposed_local(s, (2, 1, 1), 1.0 * RC)
    assert abs(res[0]["energy"].item() - ref["energy"].item()) > 1e-6 * abs(ref["energy"].item())


def test_layer_shells_order_and_counts():
    """Owned atoms keep their order in front; ghosts follow by shell; counts are per shell."""
    g = torch.Generator().manual_seed(3)
    own = torch.rand(50, 3, generator=g, dtype=torch.float64) * 10.0
    ghosts = torch.tensor([[12.0, 5, 5], [-0.5, 5, 5], [5, 5, 20.5], [23.0, 5, 5], [5, -9.5, 5], [10.0, 5, 5]],
                          dtype=torch.float64)
    lo, hi = own.min(0).values, own.max(0).values
    pos = torch.cat([own, ghosts])
    perm, L = D.layer_shells(pos, 50, (True, True, False), 5.0, 3)
    d = [max(float(lo[0] - x[0]), float(x[0] - hi[0]), float(lo[1] - x[1]), float(x[1] - hi[1]), 0.0)
         for x in ghosts]  # single-axis overshoots here; z is unsplit (distance 0 along it)
    shells = [int(np.ceil(v / (5.0 * (1 + D.SHELL_MARGIN)))) for v in d]
    keep = sorted([i for i in range(6) if shells[i] <= 3], key=lambda i: shells[i])
    assert perm.tolist() == list(range(50)) + [50 + i for i in keep]
    assert L == [50 + sum(sh <= 3 - 1 - k for sh in shells) for k in range(3)]


def test_grid_for_and_validation():
    assert D.grid_for(1) == (1, 1, 1) and D.grid_for(2) == (2, 1, 1)
    assert D.grid_for(4) == (2, 2, 1) and D.grid_for(8) == (2, 2, 2)
    with pytest.raises(ValueError):
        D.grid_for(6)
    with pytest.raises(ValueError):
        D.Decomposition(np.eye(3) * 10.0, (2, 1, 1), 6.0)  # halo longer than half the cell


def _free_port():
    with socket.socket() as sk:
        sk.bind(("127.0.0.1", 0))
        return sk.getsockname()[1]


def _gloo_rank(rank, world, port, dims):
    import torch.distributed as dist

    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world)
    try:
        s = _system()
        ref = _reference(s)
        dec = D.Decomposition(s["cell"][0], dims, NHOP * RC)
        o = _owned(dec, rank, s)
        res = D.run_dist(D.decomposed_step(dec, rank, torch.tensor(s["pos"][o], dtype=torch.float64),
                                           torch.tensor(s["Z"][o]), toy_evaluate(s["cell"][0]), want_virial=True))
        assert abs(res["energy"].item() - ref["energy"].item()) <= 1e-10 * abs(ref["energy"].item())
        np.testing.assert_allclose(res["forces"].numpy(), ref["forces"].numpy()[o], rtol=1e-9, atol=1e-10)
        np.testing.assert_allclose(res["virial"].numpy(), ref["virial"].numpy(), rtol=1e-9, atol=1e-9)
    finally:
        dist.destroy_process_group()


def test_gloo_two_ranks():
    import torch.multiprocessing as mp

    mp.spawn(_gloo_rank, args=(2, _free_port(), (2, 1, 1)), nprocs=2, join=True)


def toy_avg_evaluate(cell, use_counts=True):
    """A 2-hop potential whose messages are divided by the whole system's average in-degree
    E / N, as the sparse model's conv2 (pure_cartesian_sparse_layers.py:418).  With
    ``use_counts`` the evaluator asks decomposed_step for the per-rank (edges into owned atoms,
    owned atoms) sums (``local_counts``); without it, it uses its local graph's E / N."""
    cell_t = torch.tensor(cell, dtype=torch.float64)

    def local_counts(pos, num_local, pbc):
        _, dst, _ = ON.neighbor_list(pos.detach().numpy(), cell, RC, pbc=pbc)
        return torch.tensor([float((dst < num_local).sum()), float(num_local)], dtype=torch.float64)

    def evaluate(pos, species, num_local, pbc, totals=None):
        src, dst, S = ON.neighbor_list(pos.detach().numpy(), cell, RC, pbc=pbc)
        n = pos.shape[0]
        avg = float(totals[0] / totals[1]) if totals is not None else len(src) / n
        p = pos.detach().clone().requires_grad_(True)
        src_t, dst_t = torch.tensor(src), torch.tensor(dst)
        r = p[dst_t] - p[src_t] + torch.tensor(S, dtype=torch.float64) @ cell_t
        r.retain_grad()
        phi = (1.0 - r.norm(dim=1) / RC) ** 2
        w = 1.0 + 0.1 * species.to(torch.float64)
        m1 = torch.zeros(n, dtype=torch.float64).index_add(0, dst_t, phi * w[src_t]) / avg
        m2 = torch.zeros(n, dtype=torch.float64).index_add(0, dst_t, phi * torch.tanh(0.3 * m1[src_t])) / avg
        e = 0.01 * m2 ** 2 + 0.5 * m1 + 0.05 * m1 * m2
        E = e[:num_local].sum()
        E.backward()
        return {"energy": E.detach(), "forces": -p.grad, "atom_energy": e.detach(), "virial": r.detach().T @ r.grad}

    if use_counts:
        evaluate.local_counts = local_counts
    return evaluate


@pytest.mark.parametrize("use_counts", [True, False])
def test_whole_system_average_degree_reaches_every_rank(use_counts):
    """decomposed_step sums the evaluator's local_counts over ranks before evaluating, so a
    potential normalised by the whole system's E / N decomposes exactly; a rank's own E / N
    (truncated neighbour lists at the halo's edge) does not."""
    s = _system()
    pos = torch.tensor(s["pos"], dtype=torch.float64)
    ref = toy_avg_evaluate(s["cell"][0], use_counts=False)(pos, torch.tensor(s["Z"]), pos.shape[0], (True, True, True))
    dec = D.Decomposition(s["cell"][0], (2, 1, 1), NHOP * RC)
    ev = toy_avg_evaluate(s["cell"][0], use_counts)
    owned = [_owned(dec, r, s) for r in range(dec.world)]
    gens = [D.decomposed_step(dec, r, torch.tensor(s["pos"][o], dtype=torch.float64), torch.tensor(s["Z"][o]), ev)
            for r, o in enumerate(owned)]
    res = D.run_local(gens)
    F = np.zeros_like(s["pos"])
    for o, r in zip(owned, res):
        F[o] = r["forces"].numpy()
    rel = abs(res[0]["energy"].item() - ref["energy"].item()) / abs(ref["energy"].item())
    if use_counts:
        assert rel <= 1e-10
        np.testing.assert_allclose(F, ref["forces"].numpy(), rtol=1e-9, atol=1e-10)
    else:
        assert rel > 1e-6


@pytest.mark.parametrize("make,per_cell", [(systems.diamond_block, 8), (systems.fcc_block, 4)])
def test_lattice_blocks_tile_the_global_crystal(make, per_cell):
    """Weak-scaling blocks: each rank's block holds its cells' atoms next to its own region of the
    dims * n_cells crystal; unsplit axes are wrapped into the global cell."""
    dims, cells = (2, 2, 1), (3, 3, 3)
    blocks = [make(D.block_of(r, dims), dims, n_cells=cells, seed=r) for r in range(4)]
    L = blocks[0]["cell"][0].diagonal()
    for r, b in enumerate(blocks):
        assert b["pos"].shape[0] == per_cell * 27
        np.testing.assert_allclose(b["cell"][0].diagonal(), L)
        lo = np.asarray(D.block_of(r, dims)) * L / np.asarray(dims)
        hi = lo + L / np.asarray(dims)
        for k in range(3):
            if dims[k] > 1:  # thermal displacements stay within a fraction of a lattice constant
                assert b["pos"][:, k].min() > lo[k] - 1.0 and b["pos"][:, k].max() < hi[k] + 1.0
            else:
                assert b["pos"][:, k].min() >= 0.0 and b["pos"][:, k].max() < L[k]


def _exchange_adjoint_gen(dec, rank, pos, Z, seed):
    """Per rank: halo plan, then <x_after_exchange, y> versus <x, y_after_return>."""
    plan = yield from D.halo_exchange(dec, rank, pos, Z)
    n, G = pos.shape[0], plan.ghost_pos.shape[0]
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(n + G, 2, 3, generator=g, dtype=torch.float64)
    y = torch.randn(n + G, 2, 3, generator=g, dtype=torch.float64)
    x_owned = x[:n].clone()
    xe = x.clone()
    yield from D.exchange_ghost_rows(plan, xe, n)
    yr = y.clone()
    yield from D.return_ghost_rows(plan, yr, n)
    # owned rows are untouched by the forward exchange; ghosts were overwritten and are zero in yr
    assert torch.equal(xe[:n], x_owned) and torch.count_nonzero(yr[n:]) == 0
    lhs = yield from D.all_reduce_sum((xe * y).sum().reshape(1))
    rhs = yield from D.all_reduce_sum((x * yr).sum().reshape(1))
    # every received ghost row equals its owner's row, wherever the owner lives
    return float(lhs), float(rhs), G


@pytest.mark.parametrize("dims", [(2, 1, 1), (2, 2, 1), (2, 2, 2)])
def test_ghost_row_exchange_and_return_are_adjoint(dims):
    """The per-layer ghost-feature exchange and its gradient return satisfy <E x, y> = <x, E^T y>
    (emulated ranks in one process)."""
    s = _system()
    dec = D.Decomposition(s["cell"][0], dims, RC)
    owned = [_owned(dec, r, s) for r in range(dec.world)]
    gens = [_exchange_adjoint_gen(dec, r, torch.tensor(s["pos"][o], dtype=torch.float64), torch.tensor(s["Z"][o]),
                                  100 + r) for r, o in enumerate(owned)]
    res = D.run_local(gens)
    for lhs, rhs, G in res:
        assert G > 0
        assert abs(lhs - rhs) <= 1e-10 * max(1.0, abs(lhs))


def test_ghost_rows_carry_owner_values():
    """After the exchange every ghost row is the row of the owned atom it images."""
    s = _system()
    dec = D.Decomposition(s["cell"][0], (2, 2, 1), RC)
    owned = [_owned(dec, r, s) for r in range(dec.world)]

    def gen(rank, o):
        pos = torch.tensor(s["pos"][o], dtype=torch.float64)
        plan = yield from D.halo_exchange(dec, rank, pos, torch.tensor(s["Z"][o]))
        rows = torch.cat([torch.tensor(o, dtype=torch.float64).unsqueeze(1),
                          torch.full((plan.ghost_pos.shape[0], 1), -1.0, dtype=torch.float64)])
        yield from D.exchange_ghost_rows(plan, rows, len(o))
        return rows[len(o):, 0].long().numpy(), plan.ghost_pos.numpy()

    for gids, gpos in D.run_local([gen(r, o) for r, o in enumerate(owned)]):
        assert (gids >= 0).all()
        # a ghost image differs from its owner's position by a lattice vector
        d = (gpos - s["pos"][gids]) @ np.linalg.inv(s["cell"][0])
        assert np.abs(d - np.round(d)).max() < 1e-9


def _gloo_exchange_rank(rank, world, port, dims):
    import torch.distributed as dist

    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world)
    try:
        s = _system()
        dec = D.Decomposition(s["cell"][0], dims, RC)
        o = _owned(dec, rank, s)
        lhs, rhs, G = D.run_dist(_exchange_adjoint_gen(dec, rank, torch.tensor(s["pos"][o], dtype=torch.float64),
                                                       torch.tensor(s["Z"][o]), 100 + rank))
        assert G > 0 and abs(lhs - rhs) <= 1e-10 * max(1.0, abs(lhs))
    finally:
        dist.destroy_process_group()


def test_gloo_ghost_row_exchange():
    import torch.multiprocessing as mp

    mp.spawn(_gloo_exchange_rank, args=(2, _free_port(), (2, 1, 1)), nprocs=2, join=True)


def _select_ghosts_brute(dec, rank, pos, bboxes):
    """Every owned atom, every image, every rank: the definition the vectorised selection follows."""
    cell = torch.tensor(dec.cell, dtype=torch.float64)
    split = torch.tensor(dec.split)
    lo, hi = bboxes[:, 0, :] - dec.halo, bboxes[:, 1, :] + dec.halo
    rows = []
    for si, S in enumerate(dec.images()):
        x = pos + torch.tensor(S, dtype=torch.float64) @ cell
        inside = (((x[:, None, :] >= lo[None]) & (x[:, None, :] <= hi[None])) | ~split[None, None, :]).all(-1)
        if S == (0, 0, 0):
            inside[:, rank] = False
        for i, d in inside.nonzero().tolist():
            rows.append((d, si, i))
    rows.sort()
    counts = [sum(1 for r in rows if r[0] == d) for d in range(bboxes.shape[0])]
    return [r[2] for r in rows], [r[1] for r in rows], counts


@pytest.mark.parametrize("dims", [(2, 1, 1), (2, 2, 1), (2, 2, 2), (3, 1, 2)])
def test_vectorised_ghost_selection_matches_definition(dims):
    s = systems.diamond_crystal(n_cells=(6, 6, 6), seed=17)
    cell = s["cell"][0]
    dec = D.Decomposition(cell, dims, 5.0)
    pos = torch.tensor(s["pos"])
    frac = s["pos"] @ np.linalg.inv(cell)
    frac -= np.floor(frac)
    owner = np.zeros(len(frac), dtype=np.int64)
    for k in range(3):
        owner = owner * dims[k] + np.floor(frac[:, k] * dims[k]).astype(np.int64)
    owned = [np.nonzero(owner == r)[0] for r in range(dec.world)]
    # the rank numbering of block_of: check the owned blocks against it, then build the boxes
    bb = torch.stack([torch.stack([pos[o].min(0).values, pos[o].max(0).values]) for o in owned])
    for r in range(dec.world):
        p = pos[owned[r]]
        got_i, got_s, got_c = D.select_ghosts(dec, r, p, bb, chunk=37)
        ref_i, ref_s, ref_c = _select_ghosts_brute(dec, r, p, bb)
        assert got_c == ref_c
        assert got_i.tolist() == ref_i and got_s.tolist() == ref_s
