"""Functional CPU restatement of the ``pure-cartesian-ictd-o3`` model (test infrastructure only).

Follows ``models/pure_cartesian_ictd_layers_o3.py`` (PureCartesianICTDO3TransformerLayer
``:535-1074``, ICTDO3E3Conv ``:298-533``) and ``models/ictd_irreps.py``
(HarmonicFullyConnectedTensorProductO3 ``:1325-1695``, HarmonicElementwiseProductO3 ``:1270-1322``):
features are blocks keyed by (l, parity); a tensor-product path (l1,p1) x (l2,p2) -> (l3,p3)
exists when l1+l2+l3 is even, p3 = p1 p2 and (l3, p3) is active, with the SO(3) coupling
tensors.  The external field enters conv1 as an extra l=1 term of the canonical-parity input
block, ``Ai[src] (x) scale * t_graph`` (``:466-502``), t = the field projected on the ICTD l=1
harmonic basis (PhysicalTensorICTDEmbedding, ``pure_cartesian_ictd_layers.py:155-340``).
Physical-tensor heads are bias-free linear maps of the readout blocks summed per graph
(``:1010-1044``).  Pinned by ``tests/golden/ictd_o3_*.npz`` (generated from the reference).
"""

from __future__ import annotations

import math
from typing import Dict, List, Tuple

import torch
import torch.nn.functional as Fnn

from oracle import ictd_tables as T
from oracle.ictd_model import _layer_norm, _mlp, _scatter_sum, main_net  # noqa: F401
from oracle.radial import soft_one_hot_linspace

Key = Tuple[int, int]
ACTIVE: List[Key] = [(0, 1), (1, 1), (1, -1), (2, 1)]  # 0e, 1e, 1o, 2e


def key_str(k: Key) -> str:
    return f"{k[0]}{'e' if k[1] > 0 else 'o'}"


def o3_paths(active: List[Key], lmax: int = 2):
    """Path list (l1,p1,l2,p2,l3,p3) in the reference enumeration order (``ictd_irreps.py:1356-1366``)."""
    act = set(active)
    out = []
    for l1, p1 in active:
        for l2, p2 in active:
            for l3 in range(abs(l1 - l2), min(l1 + l2, lmax) + 1):
                if (l1 + l2 + l3) % 2 == 1 or (l3, p1 * p2) not in act:
                    continue
                out.append((l1, p1, l2, p2, l3, p1 * p2))
    return out


def o3_fctp(paths, x1: Dict[Key, torch.Tensor], x2: Dict[Key, torch.Tensor], weight, gates, active):
    """HarmonicFullyConnectedTensorProductO3.forward with internal weights and per-path gates:
    out[(l3,p3)] += gate_p * W_p . (CG_p contraction of a (x) b)."""
    sample = next(iter(x1.values()))
    E = sample.shape[0]
    mul_out = weight.shape[1]
    out = {k: torch.zeros(E, mul_out, 2 * k[0] + 1, dtype=sample.dtype) for k in active}
    for p, (l1, p1, l2, p2, l3, p3) in enumerate(paths):
        a, b = x1.get((l1, p1)), x2.get((l2, p2))
        if a is None or b is None:
            continue
        C = T.normalized_cg(l1, l2, l3).to(sample.dtype)
        y = torch.einsum("eim,ejn,mnk,oij->eok", a, b, C, weight[p])
        out[(l3, p3)] = out[(l3, p3)] + y * gates[:, p, None, None]
    return out


def split_o3(x, C, active):
    out, idx = {}, 0
    for k in active:
        d = C * (2 * k[0] + 1)
        out[k] = x[:, idx:idx + d].reshape(x.shape[0], C, 2 * k[0] + 1)
        idx += d
    return out


def merge_o3(blocks, active):
    return torch.cat([blocks[k].flatten(1) for k in active], dim=-1)


def field_harmonic(field: torch.Tensor) -> torch.Tensor:
    """(B, 3) Cartesian vectors -> (B, 3) l=1 ICTD harmonic components: monomial coefficients in
    ``counts_list(1)`` order projected with P_{1->1}."""
    idx = [0 if a else (1 if b else 2) for (a, b, c) in T.counts_list(1)]
    coeffs = field[:, idx]
    return coeffs @ T.projector(1, 1).to(field.dtype).T


def o3_forward(sd: Dict[str, torch.Tensor], cfg, pos, A, batch, edge_src, edge_dst, edge_shifts, cell, field,
               heads=("dipole", "polarizability")):
    """Per-atom energy (N, 1) and the physical-tensor heads {name: {l: (B, 1, 2l+1)}}."""
    dtype = pos.dtype
    C, lmax, nint = cfg.channels, cfg.lmax, cfg.num_interaction
    active = ACTIVE
    paths = o3_paths(active, lmax)
    N = pos.shape[0]
    B = cell.shape[0]
    order = torch.argsort(edge_dst, stable=True)
    src, dst, shifts = edge_src[order], edge_dst[order], edge_shifts[order].to(dtype)
    edge_vec = pos[dst] - pos[src] + torch.einsum("ni,nij->nj", shifts, cell[batch[src]])
    length = edge_vec.norm(dim=1)
    n = edge_vec / length.clamp(min=1e-8).unsqueeze(-1)
    Y = [T.direction_harmonics(n, l) for l in range(lmax + 1)]
    emb = soft_one_hot_linspace(length, 0.0, cfg.max_radius, cfg.number_of_basis, basis=cfg.function_type,
                                cutoff=True) * (cfg.number_of_basis ** 0.5)
    deg = _scatter_sum(torch.ones_like(dst), dst, N).clamp(min=1).to(dtype)

    # conv1 (:424-533)
    p = "e3_conv_emb"
    Ai = _mlp(sd, f"{p}.atom_mlp", sd[f"{p}.atom_embedding.weight"][A.long()], 2)
    O8 = Ai.shape[1]
    E = src.shape[0]
    f_in = {k: torch.zeros(E, O8, 2 * k[0] + 1, dtype=dtype) for k in active}
    for l in range(lmax + 1):
        k = (l, 1 if l % 2 == 0 else -1)
        if k in active:
            f_in[k] = Ai[src].unsqueeze(-1) * Y[l].unsqueeze(-2)
    if field is not None:
        t = field_harmonic(field.to(dtype))[batch][src].unsqueeze(-2)  # (E, 1, 3)
        scale = sd[f"{p}.external_tensor_scale_by_irrep"][active.index((1, -1))]
        f_in[(1, -1)] = f_in[(1, -1)] + (t * Ai[src].unsqueeze(-1)) * scale
    x2 = {k: torch.zeros(E, O8, 2 * k[0] + 1, dtype=dtype) for k in active}
    x2[(0, 1)] = Ai[dst].unsqueeze(-1)
    gates = _mlp(sd, f"{p}.fc", emb, 3)
    blocks = o3_fctp(paths, f_in, x2, sd[f"{p}.tp2.weight"], gates, active)
    feats = [_scatter_sum(merge_o3(blocks, active), dst, N) / deg.unsqueeze(-1)]

    # conv2..N (:956-973)
    for k in range(nint - 1):
        gates = _mlp(sd, f"fc2_layers.{k}", emb, 3)
        x1 = split_o3(feats[-1], C, active)
        x1e = {key: blk[src] for key, blk in x1.items()}
        Yd = {}
        for l in range(lmax + 1):
            key = (l, 1 if l % 2 == 0 else -1)
            if key in active:
                Yd[key] = Y[l].unsqueeze(-2)
        blocks = o3_fctp(paths, x1e, Yd, sd[f"tp2_layers.{k}.weight"], gates, active)
        feats.append(_scatter_sum(merge_o3(blocks, active), dst, N) / deg.unsqueeze(-1))

    # readout (:975-1066): Gram invariants of the flat split of the concatenation
    nC = C * nint
    xb = split_o3(torch.cat(feats, dim=-1), nC, active)
    S = (nint - 1) * cfg.invariant_channels
    scalars = torch.zeros(N, S, dtype=dtype)
    for key in active:
        t = xb[key]
        gram = torch.einsum("ncm,ndm->ncd", t, t) / math.sqrt(2 * key[0] + 1)
        scalars = scalars + torch.einsum("ocd,ncd->no", sd[f"W_read.{key_str(key)}"], gram)
    splits = [split_o3(f, C, active) for f in feats]
    Tb = {key: torch.cat([s[key] for s in splits], dim=-2) for key in active}
    Tb[(0, 1)] = torch.cat([Tb[(0, 1)], scalars.unsqueeze(-1)], dim=-2)
    p5 = [(Tb[key] * Tb[key]).sum(dim=-1) * T.normalized_cg(key[0], key[0], 0, "norm")[0, 0, 0].item()
          for key in active]
    proj = main_net(sd, "proj_total", torch.cat(p5, dim=-1), len(cfg.embed_size))
    e = (proj * sd["weighted_sum.weights"]).sum(dim=-1, keepdim=True)

    out_heads = {}
    spec = {"dipole": [(1, -1)], "polarizability": [(0, 1), (2, 1)]}
    for name in heads:
        res = {}
        for key in spec[name]:
            W = sd[f"physical_tensor_heads.{name}.{key[0]}.weight"]  # (1, nC)
            y = torch.einsum("oc,ncm->nom", W, xb[key])
            res[key[0]] = torch.zeros(B, y.shape[1], y.shape[2], dtype=dtype).index_add(0, batch, y)
        out_heads[name] = res
    return e, out_heads


def o3_energy_forces(sd, cfg, pos, A, batch, edge_src, edge_dst, edge_shifts, cell, field):
    pos = pos.detach().clone().requires_grad_(True)
    e, heads = o3_forward(sd, cfg, pos, A, batch, edge_src, edge_dst, edge_shifts, cell, field)
    B = cell.shape[0]
    Eg = torch.zeros(B, dtype=pos.dtype).index_add(0, batch, e.squeeze(-1))
    (g,) = torch.autograd.grad(Eg.sum(), [pos])
    return {"energy": Eg.detach(), "forces": -g, "atom_energy": e.detach().squeeze(-1),
            "dipole": heads["dipole"][1].detach(), "polar0": heads["polarizability"][0].detach(),
            "polar2": heads["polarizability"][2].detach()}
