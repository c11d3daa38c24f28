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


def _check(sysd, r=5.0):
    dev = torch.device("cuda")
    pos = torch.tensor(sysd["pos"], device=dev)
    cell = torch.tensor(sysd["cell"], device=dev)
    b = sysd["batch"]
    fp = np.concatenate([[0], np.cumsum(np.bincount(b, minlength=sysd["cell"].shape[0]))])
    src, dst, S = radius_graph_pbc(pos, r, cell, pbc=sysd["pbc"], frame_ptr=fp)
    torch.cuda.synchronize()
    os_, od, oS = ON.batched_neighbor_list(sysd["pos"], b, sysd["cell"], r, sysd["pbc"])
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
