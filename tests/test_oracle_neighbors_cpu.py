"""CPU checks of the neighbour-list oracle's per-source cap (``max_num_neighbors`` of
``radius_graph_pbc_gpu``, ``utils/graph_utils.py:192, 240``)."""

import numpy as np

from fsctep_b200 import systems
from oracle import neighbors as ON


def _chain(n=8):
    pos = np.zeros((n, 3))
    pos[:, 0] = np.arange(n, dtype=np.float64) + 10.0
    return pos, np.eye(3) * 40.0


def test_known_answer_chain():
    """Atoms 1 A apart on a line, cutoff 2.5, cap 2: the query visits j = i-2, i-1, i (self),
    i+1, i+2 in that order and keeps its first two hits."""
    pos, cell = _chain()
    src, dst, S = ON.neighbor_list(pos, cell, 2.5, pbc=(False, False, False), max_num_neighbors=2)
    got = sorted(zip(src.tolist(), dst.tolist()))
    want = [(0, 1), (1, 0)] + [(i, j) for i in range(2, 8) for j in (i - 2, i - 1)]
    assert got == sorted(want)
    assert not S.any()


def test_large_cap_changes_nothing():
    s = systems.water_box(n_side=3, box=9.3, seed=3)
    full = ON.neighbor_list(s["pos"], s["cell"][0], 5.0, s["pbc"])
    capped = ON.neighbor_list(s["pos"], s["cell"][0], 5.0, s["pbc"], max_num_neighbors=10_000)
    for a, b in zip(full, capped):
        np.testing.assert_array_equal(a, b)


def test_cap_keeps_the_lowest_candidates_per_image():
    s = systems.diamond_crystal(n_cells=(2, 2, 2), seed=4)
    cell = s["cell"][0]
    full = ON.neighbor_list(s["pos"], cell, 5.0, s["pbc"])
    src, dst, S = ON.neighbor_list(s["pos"], cell, 5.0, s["pbc"], max_num_neighbors=3, chunk=7)
    assert 0 < src.shape[0] < full[0].shape[0]
    key = lambda a, b, c: {(int(i), int(j), tuple(int(x) for x in t)) for i, j, t in zip(a, b, c)}  # noqa: E731
    kept, every = key(src, dst, S), key(*full)
    assert kept <= every
    for i in range(s["pos"].shape[0]):
        for t in {e[2] for e in every if e[0] == i}:
            cand = sorted(j for (a, j, u) in every if a == i and u == t)
            if t == (0, 0, 0):  # the self pair is the query's hit at j == i
                cand = sorted(cand + [i])
            first = [j for j in cand[:3] if not (t == (0, 0, 0) and j == i)]
            assert sorted(j for (a, j, u) in kept if a == i and u == t) == first
