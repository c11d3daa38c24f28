"""Seeded synthetic systems with the shapes of the benchmark configurations.

No public dataset is involved: every system is generated from a seed with the
sizes, densities and species mix named by the benchmark configurations.

* ``random_frames``  -- config 1: frames of uniform random atoms in a cubic box,
  rejection below a minimum (minimum-image) pair distance, species uniform.
* ``water_box``      -- config 2: H2O molecules, O on a jittered grid, O-H 0.96 A,
  H-O-H 104.5 deg, random orientations.
* ``organic_molecules`` -- config 3: non-periodic random bonded chains, C:H:N:O = 3:5:1:1.
* ``diamond_crystal`` -- config 4: diamond lattice with Gaussian displacements.
* ``fcc_crystal``    -- config 5: FCC lattice with Gaussian displacements.

All return a dict with ``pos`` (N,3) float64, ``Z`` (N,) int64, ``batch`` (N,)
int64, ``cell`` (B,3,3) float64 (rows are lattice vectors) and ``pbc``.
"""

from __future__ import annotations

import math

import numpy as np


def _system(pos, Z, batch, cells, pbc=(True, True, True)):
    return {"pos": np.ascontiguousarray(pos, dtype=np.float64), "Z": np.asarray(Z, dtype=np.int64),
            "batch": np.asarray(batch, dtype=np.int64), "cell": np.asarray(cells, dtype=np.float64),
            "pbc": tuple(bool(p) for p in pbc)}


def random_frames(n_frames=8, n_atoms=96, box=10.0, min_dist=0.9, species=(1, 6, 8), seed=0):
    rng = np.random.default_rng(seed)
    pos_all, Z_all, b_all = [], [], []
    for f in range(n_frames):
        pts = np.zeros((0, 3))
        while pts.shape[0] < n_atoms:
            cand = rng.uniform(0.0, box, size=3)
            if pts.shape[0]:
                d = pts - cand
                d -= box * np.round(d / box)
                if np.min(np.einsum("ij,ij->i", d, d)) < min_dist * min_dist:
                    continue
            pts = np.vstack([pts, cand])
        pos_all.append(pts)
        Z_all.append(rng.choice(np.asarray(species), size=n_atoms))
        b_all.append(np.full(n_atoms, f))
    cells = np.stack([np.eye(3) * box for _ in range(n_frames)])
    return _system(np.concatenate(pos_all), np.concatenate(Z_all), np.concatenate(b_all), cells)


def _random_rotation(rng):
    q = rng.normal(size=4)
    q /= np.linalg.norm(q)
    w, x, y, z = q
    return np.array([[1 - 2 * (y * y + z * z), 2 * (x * y - z * w), 2 * (x * z + y * w)],
                     [2 * (x * y + z * w), 1 - 2 * (x * x + z * z), 2 * (y * z - x * w)],
                     [2 * (x * z - y * w), 2 * (y * z + x * w), 1 - 2 * (x * x + y * y)]])


def water_box(n_side=10, box=31.0, sigma=0.3, seed=0):
    rng = np.random.default_rng(seed)
    a = box / n_side
    g = (np.arange(n_side) + 0.5) * a
    O = np.stack(np.meshgrid(g, g, g, indexing="ij"), axis=-1).reshape(-1, 3)
    O = O + rng.normal(scale=sigma, size=O.shape)
    half = math.radians(104.5) / 2
    h1 = 0.96 * np.array([math.sin(half), math.cos(half), 0.0])
    h2 = 0.96 * np.array([-math.sin(half), math.cos(half), 0.0])
    pos, Z = [], []
    for o in O:
        R = _random_rotation(rng)
        pos.extend([o, o + R @ h1, o + R @ h2])
        Z.extend([8, 1, 1])
    pos = np.mod(np.asarray(pos), box)
    return _system(pos, Z, np.zeros(len(Z)), (np.eye(3) * box)[None])


def organic_molecules(n_mol=256, min_atoms=10, max_atoms=30, seed=0, min_dist=0.9,
                      bond=(1.1, 1.5), spacing=100.0):
    """Random bonded chains; each molecule in its own far-apart frame (non-periodic)."""
    rng = np.random.default_rng(seed)
    elems = np.array([6] * 3 + [1] * 5 + [7] + [8])
    pos_all, Z_all, b_all = [], [], []
    for m in range(n_mol):
        n = int(rng.integers(min_atoms, max_atoms + 1))
        pts = [np.zeros(3)]
        while len(pts) < n:
            base = pts[int(rng.integers(0, len(pts)))]
            v = rng.normal(size=3)
            cand = base + v / np.linalg.norm(v) * rng.uniform(*bond)
            if np.min(np.linalg.norm(np.asarray(pts) - cand, axis=1)) < min_dist:
                continue
            pts.append(cand)
        pts = np.asarray(pts)
        pos_all.append(pts - pts.mean(axis=0) + spacing / 2)
        Z_all.append(rng.choice(elems, size=n))
        b_all.append(np.full(n, m))
    cells = np.stack([np.eye(3) * spacing for _ in range(n_mol)])
    return _system(np.concatenate(pos_all), np.concatenate(Z_all), np.concatenate(b_all), cells,
                   pbc=(False, False, False))


def _lattice(basis, n_cells, a, sigma, seed, Z):
    rng = np.random.default_rng(seed)
    nx, ny, nz = n_cells
    ii, jj, kk = np.meshgrid(np.arange(nx), np.arange(ny), np.arange(nz), indexing="ij")
    origins = np.stack([ii, jj, kk], axis=-1).reshape(-1, 1, 3).astype(np.float64)
    pos = ((origins + np.asarray(basis)[None]) * a).reshape(-1, 3)
    pos = pos + rng.normal(scale=sigma, size=pos.shape)
    L = np.array([nx, ny, nz], dtype=np.float64) * a
    pos = np.mod(pos, L)
    return _system(pos, np.full(pos.shape[0], Z), np.zeros(pos.shape[0]), np.diag(L)[None])


DIAMOND_BASIS = [(0, 0, 0), (0, .5, .5), (.5, 0, .5), (.5, .5, 0),
                 (.25, .25, .25), (.25, .75, .75), (.75, .25, .75), (.75, .75, .25)]
FCC_BASIS = [(0, 0, 0), (0, .5, .5), (.5, 0, .5), (.5, .5, 0)]


def diamond_crystal(n_cells=(50, 50, 50), a=5.43, sigma=0.08, seed=0, Z=14):
    """Diamond lattice; 50^3 conventional cells x 8 atoms = 1,000,000 atoms."""
    return _lattice(DIAMOND_BASIS, n_cells, a, sigma, seed, Z)


def diamond_block(block, dims, n_cells=(50, 50, 50), a=5.43, sigma=0.08, seed=0, Z=14):
    """One rank's block of a diamond crystal of dims * n_cells conventional cells (spatial
    decomposition, weak scaling: n_cells per rank).  Positions are wrapped into the global cell
    only along unsplit axes (dims == 1); along split axes a displaced atom stays next to its
    own block.  Returns the block's atoms and the global cell."""
    return _lattice_block(DIAMOND_BASIS, block, dims, n_cells, a, sigma, seed, Z)


def fcc_block(block, dims, n_cells=(50, 50, 25), a=3.61, sigma=0.1, seed=0, Z=29):
    """One rank's block of an FCC crystal of dims * n_cells cells (as :func:`diamond_block`)."""
    return _lattice_block(FCC_BASIS, block, dims, n_cells, a, sigma, seed, Z)


def _lattice_block(basis, block, dims, n_cells, a, sigma, seed, Z):
    rng = np.random.default_rng(seed)
    nx, ny, nz = n_cells
    ii, jj, kk = np.meshgrid(np.arange(nx), np.arange(ny), np.arange(nz), indexing="ij")
    origins = np.stack([ii, jj, kk], axis=-1).reshape(-1, 1, 3).astype(np.float64)
    origins = origins + (np.asarray(block, dtype=np.float64) * np.asarray(n_cells))[None, None, :]
    pos = ((origins + np.asarray(basis)[None]) * a).reshape(-1, 3)
    pos = pos + rng.normal(scale=sigma, size=pos.shape)
    L = np.asarray(n_cells, dtype=np.float64) * np.asarray(dims) * a
    for k in range(3):
        if dims[k] == 1:
            pos[:, k] = np.mod(pos[:, k], L[k])
    return _system(pos, np.full(pos.shape[0], Z), np.zeros(pos.shape[0]), np.diag(L)[None])


def fcc_crystal(n_cells=(50, 50, 25), a=3.61, sigma=0.1, seed=0, Z=29):
    """FCC lattice; 50x50x25 cells x 4 atoms = 250,000 atoms."""
    return _lattice(FCC_BASIS, n_cells, a, sigma, seed, Z)
