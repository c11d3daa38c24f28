"""GPU neighbour list: bit-exact edge sets against the CPU oracle."""

import numpy as np
import pytest
import torch

import golden_io
import gpu_util as U
from fsctep_b200 import systems
from fsctep_b200.neighbors import radius_graph_pbc
from oracle import neighbors as ON

pytestmark = [pytest.mark.gpu, U.needs_gpu]


def _check(sysd, r=5.0, cap=None):
    dev = torch.device("cuda")
    pos = torch.tensor(sysd["pos"], device=dev)
    cell = torch.tensor(sysd["cell"], device=dev)
    b = sysd["batch"]
    fp = np.concatenate([[0], np.cumsum(np.bincount(b, minlength=sysd["cell"].shape[0]))])
    src, dst, S = radius_graph_pbc(pos, r, cell, max_num_neighbors=cap, pbc=sysd["pbc"], frame_ptr=fp)
    torch.cuda.synchronize()
    os_, od, oS = ON.batched_neighbor_list(sysd["pos"], b, sysd["cell"], r, sysd["pbc"], max_num_neighbors=cap)
    np.testing.assert_array_equal(dst.cpu().numpy(), od)
    np.testing.assert_array_equal(src.cpu().numpy(), os_)
    np.testing.assert_array_equal(S.cpu().numpy().astype(np.int64), oS)


@pytest.mark.parametrize("tag", ["a", "b", "c"])
def test_golden_frames(tag):
    _, _, c = golden_io.model_case(tag)
    _check({k: c[k] for k in ("pos", "batch", "cell")} | {"pbc": tuple(bool(x) for x in c["pbc"])})


def test_cell_list_diamond():
    _check(systems.diamond_crystal(n_cells=(6, 6, 6), seed=3))


def test_cell_list_water():
    _check(systems.water_box(n_side=10, box=31.0, seed=4))


def test_small_box_fewer_than_three_cells():
    _check(systems.fcc_crystal(n_cells=(16, 16, 3), seed=5))  # z: 10.8 A -> 2 cells, cell list path


def test_nonperiodic_molecules():
    _check(systems.organic_molecules(n_mol=8, seed=6))


def test_positions_outside_box_fall_back_to_all_pairs():
    s = systems.diamond_crystal(n_cells=(6, 6, 6), seed=7)
    s["pos"] = s["pos"] + np.array([0.5, -0.3, 0.0])  # some atoms leave [0, L)
    _check(s)


def test_cell_list_slab_open_z():
    s = systems.diamond_crystal(n_cells=(6, 6, 6), seed=8)
    s["pbc"] = (True, True, False)
    _check(s)


def test_cell_list_open_cluster():
    s = systems.diamond_crystal(n_cells=(6, 6, 5), seed=9)
    s["pbc"] = (False, False, False)
    _check(s)


def test_cell_list_split_axis_with_ghost_images():
    """Layout of a spatial-decomposition rank: open along x with atoms outside [0, L), periodic y, z."""
    s = systems.diamond_crystal(n_cells=(8, 5, 5), seed=10)
    s["pos"] = s["pos"] + np.array([-7.5, 0.0, 0.0])
    s["pbc"] = (False, True, True)
    _check(s)


def _dense_cluster(n=300, box=8.0, seed=12):
    rng = np.random.default_rng(seed)
    pts = []
    while len(pts) < n:
        p = rng.uniform(0.0, box, 3)
        if all(np.sum((p - q) ** 2) >= 0.81 for q in pts):
            pts.append(p)
    pos = np.asarray(pts) + 20.0
    return systems._system(pos, np.ones(n, dtype=np.int64), np.zeros(n, dtype=np.int64), (np.eye(3) * 60.0)[None],
                           pbc=(False, False, False))


@pytest.mark.parametrize("cap", [100, 7])
def test_cap_dense_cluster(cap):
    """More than 100 candidates per source: the reference's default cap bites."""
    s = _dense_cluster()
    _, od, _ = ON.batched_neighbor_list(s["pos"], s["batch"], s["cell"], 5.0, s["pbc"])
    assert np.bincount(od).max() > 100
    _check(s, cap=cap)


@pytest.mark.parametrize("cap", [3, 20])
def test_cap_cell_list_and_images(cap):
    _check(systems.diamond_crystal(n_cells=(6, 6, 6), seed=13), cap=cap)
    _check(systems.fcc_crystal(n_cells=(3, 3, 3), seed=14), cap=cap)  # all-pairs path, 27 images


def test_cap_known_answer_chain():
    pos = np.zeros((8, 3))
    pos[:, 0] = np.arange(8, dtype=np.float64) + 10.0
    dev = torch.device("cuda")
    src, dst, S = radius_graph_pbc(torch.tensor(pos, device=dev), 2.5, torch.tensor(np.eye(3) * 40.0, device=dev)[None],
                                   max_num_neighbors=2, pbc=(False, False, False))
    got = sorted(zip(src.cpu().tolist(), dst.cpu().tolist()))
    assert got == sorted([(0, 1), (1, 0)] + [(i, j) for i in range(2, 8) for j in (i - 2, i - 1)])


def test_default_cap_is_inactive_on_the_benchmark_lattices():
    """Diamond Si and FCC Cu at 5 A stay far below 100 candidates per source and image."""
    for s in (systems.diamond_crystal(n_cells=(4, 4, 4), seed=15), systems.fcc_crystal(n_cells=(4, 4, 4), seed=16)):
        dev = torch.device("cuda")
        pos, cell = torch.tensor(s["pos"], device=dev), torch.tensor(s["cell"], device=dev)
        a = radius_graph_pbc(pos, 5.0, cell)
        b = radius_graph_pbc(pos, 5.0, cell, max_num_neighbors=None)
        for x, y in zip(a, b):
            assert torch.equal(x, y)
