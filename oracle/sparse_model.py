"""Functional CPU restatement of the ``pure-cartesian-sparse`` model (test infrastructure only).

Follows ``models/pure_cartesian_sparse_layers.py`` (PureCartesianSparseTransformerLayer
``:459-855``, PureCartesianSparseE3Conv ``:134-330``, PureCartesianSparseE3Conv2 ``:333-421``,
PureCartesianSparseInvariantBilinear ``:424-456``) and ``models/pure_cartesian.py``
(PureCartesianTensorProductO3Sparse ``:736-929`` with ``max_rank_other=1``, ``k_policy="k0"``,
``allow_epsilon=False``, ``assume_pseudo_zero=True``; ``_enumerate_paths_sparse`` ``:353-418``;
``edge_rank_powers`` ``:292-317``; the 0e elementwise product ``:144-196``).

With those options every path is a plain outer product (no delta or epsilon contraction) of a
rank-L1 tensor with a rank-L2 tensor, Lout = L1 + L2 <= Lmax, min(L1, L2) <= 1, and the
pseudotensor half of every feature is identically zero, so only true tensors are carried here.
Features are kept per rank L as (N, C, 3^L) with the reference's row-major flattening of the
Cartesian indices.  Pinned by ``tests/golden/sparse_*.npz`` (generated from the reference).
"""

from __future__ import annotations

import math
from typing import Dict, List, Tuple

import torch

from oracle.ictd_model import _mlp, _scatter_sum, main_net
from oracle.radial import soft_one_hot_linspace


def sparse_paths(lmax: int) -> List[Tuple[int, int, int]]:
    """(L1, L2, Lout) in the reference enumeration order (k0 policy, no epsilon)."""
    out = []
    for L1 in range(lmax + 1):
        for L2 in range(lmax + 1):
            if min(L1, L2) > 1 or L1 + L2 > lmax:
                continue
            out.append((L1, L2, L1 + L2))
    return out


def rank_powers(n: torch.Tensor, lmax: int) -> List[torch.Tensor]:
    """n^{(x)L} flattened row-major: (E, 3^L), L = 0..lmax."""
    E = n.shape[0]
    out = [torch.ones(E, 1, dtype=n.dtype)]
    for L in range(1, lmax + 1):
        out.append((out[-1].unsqueeze(-1) * n.unsqueeze(-2)).flatten(1))
    return out


def sparse_tp(paths, x1: List[torch.Tensor], x2: List[torch.Tensor], W: torch.Tensor, cout: int):
    """Per-edge weights W (E, P*cout*C1*C2): out[Lout][e, c, (i, j)] +=
    sum_{a,b} W_p[e, c, a, b] x1[L1][e, a, i] x2[L2][e, b, j]."""
    E = W.shape[0]
    C1, C2 = x1[0].shape[1], x2[0].shape[1]
    lmax = max(p[2] for p in paths)
    out = [torch.zeros(E, cout, 3 ** L, dtype=W.dtype) for L in range(lmax + 1)]
    off = 0
    for L1, L2, Lo in paths:
        Wp = W[:, off:off + cout * C1 * C2].reshape(E, cout, C1, C2)
        off += cout * C1 * C2
        ab = torch.einsum("eai,ebj->eabij", x1[L1], x2[L2]).reshape(E, C1, C2, 3 ** Lo)
        out[Lo] = out[Lo] + torch.einsum("ecab,eabk->eck", Wp, ab)
    return out


def sparse_atom_energy(sd: Dict[str, torch.Tensor], cfg, pos, A, batch, edge_src, edge_dst, edge_shifts, cell):
    dtype = pos.dtype
    C, lmax, nint = cfg.channels, cfg.lmax, cfg.num_interaction
    paths = sparse_paths(lmax)
    N = pos.shape[0]
    order = torch.argsort(edge_dst, stable=True)
    src, dst, shifts = edge_src[order], edge_dst[order], edge_shifts[order].to(dtype)
    edge_vec = pos[dst] - pos[src] + torch.einsum("ni,nij->nj", shifts, cell[batch[src]])
    length = edge_vec.norm(dim=1)
    n = edge_vec / length.clamp(min=1e-8).unsqueeze(-1)
    npow = rank_powers(n, lmax)
    emb = soft_one_hot_linspace(length, 0.0, cfg.max_radius, cfg.number_of_basis, basis=cfg.function_type,
                                cutoff=True) * (cfg.number_of_basis ** 0.5)
    E = src.shape[0]

    # conv1 (:265-330): x1 = Ai[src] (x) n^L, x2 = Ai[dst] (rank 0), mean over neighbours
    p = "e3_conv_emb"
    Ai = _mlp(sd, f"{p}.atom_mlp", sd[f"{p}.atom_embedding.weight"][A.long()], 2)
    x1 = [Ai[src].unsqueeze(-1) * npow[L].unsqueeze(-2) for L in range(lmax + 1)]
    x2 = [Ai[dst].unsqueeze(-1)] + [torch.zeros(E, Ai.shape[1], 3 ** L, dtype=dtype) for L in range(1, lmax + 1)]
    W = _mlp(sd, f"{p}.fc", emb, 3)
    blocks = sparse_tp(paths, x1, x2, W, C)
    deg = _scatter_sum(torch.ones_like(dst), dst, N).clamp(min=1).to(dtype)
    feats = [[_scatter_sum(b, dst, N) / deg.view(-1, 1, 1) for b in blocks]]

    # conv2..N (:397-421): x1 = f[src], x2 = n^L (C2 = 1), sum / (E / N)
    avg = max(E / max(N, 1), 1e-8)
    for k in range(1, nint):
        W = _mlp(sd, f"e3_conv_layers.{k}.fc", emb, 3)
        x1 = [f[src] for f in feats[-1]]
        x2 = [t.unsqueeze(-2) for t in npow]
        blocks = sparse_tp(paths, x1, x2, W, C)
        feats.append([_scatter_sum(b, dst, N) / avg for b in blocks])

    # readout (:823-838): bilinear invariants of the channel concatenation, 0e products
    S = (nint - 1) * cfg.invariant_channels
    comb = [torch.cat([f[L] for f in feats], dim=1) for L in range(lmax + 1)]  # (N, nC, 3^L)
    f3 = torch.zeros(N, S, dtype=dtype)
    for L in range(lmax + 1):
        gram = torch.einsum("ncm,ndm->ncd", comb[L], comb[L]) / math.sqrt(3 ** L)
        f3 = f3 + torch.einsum("ocd,ncd->no", sd[f"product_3.W.{L}"], gram)
    invs = [torch.cat([(f[L] * f[L]).sum(-1) / math.sqrt(3 ** L) for L in range(lmax + 1)], dim=-1) for f in feats]
    f5 = torch.cat(invs + [f3 * f3], dim=-1)
    proj = main_net(sd, "proj_total", f5, len(cfg.embed_size))
    return (proj * sd["weighted_sum.weights"]).sum(dim=-1, keepdim=True)


def sparse_energy_forces_stress(sd, cfg, pos, A, batch, edge_src, edge_dst, edge_shifts, cell, want_stress=True):
    dtype = pos.dtype
    pos = pos.detach().clone().requires_grad_(True)
    nb = cell.shape[0]
    strain = torch.zeros(nb, 3, 3, dtype=dtype, requires_grad=True)
    D = torch.eye(3, dtype=dtype) + 0.5 * (strain + strain.transpose(-1, -2))
    pos_in = torch.einsum("ni,nij->nj", pos, D[batch])
    cell_in = torch.bmm(cell.to(dtype), D)
    e = sparse_atom_energy(sd, cfg, pos_in, A, batch, edge_src, edge_dst, edge_shifts, cell_in)
    Eg = torch.zeros(nb, dtype=dtype).index_add(0, batch, e.squeeze(-1))
    gp, gs = torch.autograd.grad(Eg.sum(), [pos, strain])
    out = {"energy": Eg.detach(), "forces": -gp, "atom_energy": e.detach().squeeze(-1)}
    if want_stress:
        out["stress"] = gs / torch.abs(torch.det(cell.to(dtype))).view(-1, 1, 1)
    return out
