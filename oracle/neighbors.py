"""CPU neighbour-list oracle (test infrastructure only).

Restates the semantics of ``radius_graph_pbc_gpu`` (``utils/graph_utils.py:192-258``):

* image shifts S in {-1,0,1} on every periodic axis (``{0}`` on open axes), in the
  order of ``torch.cartesian_prod`` (``:215-222``);
* shift vector ``S @ cell`` with lattice vectors as rows (``:224-236``);
* a pair (src=i, dst=j, S) is an edge when ``|(pos[j] + S@cell) - pos[i]| < r``
  (torch_cluster ``radius(pos + S@cell, pos, r)``: query ``i`` in ``pos``, neighbour
  ``j`` in the shifted copy, ``:240-242``), excluding ``i == j`` at ``S == 0``
  (``:244-246``);
* with ``max_num_neighbors`` given, the reference's per-query cap (``:192, 240``): the
  published algorithm of torch_cluster's CUDA ``radius`` kernel (torch_cluster is a dependency
  that is not vendored) visits the candidates ``j`` of query ``i`` in ascending index order and
  stops after ``max_num_neighbors`` hits, so per image shift only the first hits survive; the
  self pair at ``S == 0`` is one of them and is removed afterwards.

Arithmetic is float64 in one fixed order, which the CUDA builder reproduces without
FMA contraction so that both produce the same edge set bit for bit:
``shift_c = (S0*cell[0,c] + S1*cell[1,c]) + S2*cell[2,c]``,
``d_c = (pos[j,c] + shift_c) - pos[i,c]``, ``r2 = (d_x*d_x + d_y*d_y) + d_z*d_z``,
edge iff ``r2 < r*r``.  Output order is canonical: by dst, then src, then shift
(lexicographic on (S0,S1,S2)).
"""

from __future__ import annotations

import itertools

import numpy as np


def image_shifts(pbc=(True, True, True)) -> np.ndarray:
    axes = [(-1, 0, 1) if p else (0,) for p in pbc]
    return np.array(list(itertools.product(*axes)), dtype=np.int64)


def shift_vectors(shifts: np.ndarray, cell: np.ndarray) -> np.ndarray:
    s = shifts.astype(np.float64)
    c = np.asarray(cell, dtype=np.float64)
    return (s[:, 0:1] * c[0][None, :] + s[:, 1:2] * c[1][None, :]) + s[:, 2:3] * c[2][None, :]


def neighbor_list(pos: np.ndarray, cell: np.ndarray, r: float, pbc=(True, True, True),
                  chunk: int = 2048, max_num_neighbors: int = None):
    """Brute-force O(27 N^2) neighbour list; returns (src, dst, shifts) int64, canonical order."""
    pos = np.asarray(pos, dtype=np.float64)
    n = pos.shape[0]
    S = image_shifts(pbc)
    sv = shift_vectors(S, cell)
    r2max = np.float64(r) * np.float64(r)
    srcs, dsts, sids = [], [], []
    for k in range(S.shape[0]):
        shifted = pos + sv[k][None, :]
        zero = not S[k].any()
        hits = np.zeros(n, dtype=np.int64)  # hits of each query so far in this image (self included)
        for j0 in range(0, n, chunk):
            pj = shifted[j0:j0 + chunk]                     # neighbours j
            d = pj[None, :, :] - pos[:, None, :]            # (i, j, 3)
            r2 = (d[..., 0] * d[..., 0] + d[..., 1] * d[..., 1]) + d[..., 2] * d[..., 2]
            m = r2 < r2max
            if max_num_neighbors is not None:
                rank = hits[:, None] + np.cumsum(m, axis=1)  # 1-based hit number of (i, j)
                hits += m.sum(axis=1)
                m &= rank <= max_num_neighbors
            ii, jj = np.nonzero(m)
            jj = jj + j0
            if zero:
                keep = ii != jj
                ii, jj = ii[keep], jj[keep]
            srcs.append(ii)
            dsts.append(jj)
            sids.append(np.full(ii.shape, k, dtype=np.int64))
    src = np.concatenate(srcs) if srcs else np.zeros(0, np.int64)
    dst = np.concatenate(dsts) if dsts else np.zeros(0, np.int64)
    sid = np.concatenate(sids) if sids else np.zeros(0, np.int64)
    order = np.lexsort((sid, src, dst))
    return src[order].astype(np.int64), dst[order].astype(np.int64), S[sid[order]]


def batched_neighbor_list(pos: np.ndarray, batch: np.ndarray, cells: np.ndarray, r: float,
                          pbc=(True, True, True), max_num_neighbors: int = None):
    """Per-frame lists concatenated with global atom indices (frames independent)."""
    out_s, out_d, out_S = [], [], []
    for g in range(cells.shape[0]):
        idx = np.nonzero(batch == g)[0]
        s, d, S = neighbor_list(pos[idx], cells[g], r, pbc, max_num_neighbors=max_num_neighbors)
        out_s.append(idx[s])
        out_d.append(idx[d])
        out_S.append(S)
    src = np.concatenate(out_s)
    dst = np.concatenate(out_d)
    S = np.concatenate(out_S)
    order = np.lexsort((S[:, 2], S[:, 1], S[:, 0], src, dst))
    return src[order], dst[order], S[order]
