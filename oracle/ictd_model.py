"""Functional CPU restatement of the ``pure-cartesian-ictd`` model (test infrastructure only).

Follows ``models/pure_cartesian_ictd_layers_full.py`` (PureCartesianICTDTransformerLayer,
ICTDIrrepsE3Conv) and ``models/ictd_irreps.py`` (HarmonicFullyConnectedTensorProduct
PyTorch fast path ``:1003-1133``, HarmonicElementwiseProduct 0e path ``:697-703``),
``models/mlp.py`` (MainNet ``:8-66``, RobustScalarWeightedSum ``:117-133``) and the
force/stress conventions of ``evaluation/calculator.py:152-159`` (F = -dE/dpos) and
``training/trainer.py:1213-1310`` (sigma = (1/V) dE/d(strain), strain applied as
``pos (I + sym eps)`` and ``cell (I + sym eps)``).

The computation order is the reference's effective GPU/CPU path (outer product,
projection with the packed U_g, per-path channel mix, gate, index_add scatter, divide
by neighbour count), so this module doubles as the timed CPU baseline.  Parameters
come from a ``state_dict`` with the reference's key names.
"""

from __future__ import annotations

import math
from typing import Dict, List, Optional

import torch
import torch.nn.functional as Fnn

from oracle import ictd_tables as T
from oracle.radial import soft_one_hot_linspace


class ICTDConfig(dict):
    """Model hyper-parameters (names follow the reference constructor)."""

    DEFAULTS = dict(channels=64, lmax=2, num_interaction=3, number_of_basis=8, max_radius=5.0,
                    function_type="gaussian", output_size=8, embedding_dim=16, max_atomvalue=10,
                    invariant_channels=32, embed_size=(128, 128, 128), path_policy="full",
                    max_rank_other=None)

    def __init__(self, **kw):
        d = dict(self.DEFAULTS)
        d.update(kw)
        super().__init__(d)

    def __getattr__(self, k):
        try:
            return self[k]
        except KeyError as e:
            raise AttributeError(k) from e


class _TPTables:
    def __init__(self, lmax: int, dtype, path_policy="full", max_rank_other=None):
        self.paths = T.tp_paths(lmax, path_policy, max_rank_other)
        self.groups = T.tp_groups(self.paths)
        self.U = [u.to(dtype) for u in T.group_U(self.paths, self.groups)]


def _mlp(sd, prefix, x, n_lin):
    """nn.Sequential(Linear, SiLU, Linear, SiLU, ..., Linear) with indices 0,2,4,..."""
    for k in range(n_lin):
        x = Fnn.linear(x, sd[f"{prefix}.{2 * k}.weight"], sd[f"{prefix}.{2 * k}.bias"])
        if k < n_lin - 1:
            x = Fnn.silu(x)
    return x


def harmonic_fctp(tabs: _TPTables, lmax, x1: Dict[int, torch.Tensor], x2: Dict[int, torch.Tensor],
                  weight: torch.Tensor, gates: torch.Tensor) -> Dict[int, torch.Tensor]:
    """HarmonicFullyConnectedTensorProduct.forward, internal weights + per-path gates
    (``ictd_irreps.py:1003-1133``, PyTorch fallback branch)."""
    sample = next(iter(x1.values()))
    E = sample.shape[0]
    mul_out, i, j = weight.shape[1], weight.shape[2], weight.shape[3]
    out = {l: torch.zeros(E, mul_out, 2 * l + 1, dtype=sample.dtype) for l in range(lmax + 1)}
    for g, U in zip(tabs.groups, tabs.U):
        a, b = x1.get(g["l1"]), x2.get(g["l2"])
        if a is None or b is None:
            continue
        m1, m2 = 2 * g["l1"] + 1, 2 * g["l2"] + 1
        t = (a.unsqueeze(-2).unsqueeze(-1) * b.unsqueeze(-3).unsqueeze(-2)).reshape(E, i, j, m1 * m2)
        y = torch.matmul(t, U)  # (E, i, j, K_total)
        for p, l3, s, e in g["segments"]:
            kd = e - s
            y2 = y[..., s:e].movedim(-1, -3).reshape(E, kd, i * j)
            W2 = weight[p].reshape(mul_out, i * j)
            seg = torch.matmul(y2, W2.T).movedim(-1, -2)  # (E, o, k)
            out[l3] = out[l3] + seg * gates[:, p, None, None]
    return out


def _split(x, C, lmax):
    out, idx = {}, 0
    for l in range(lmax + 1):
        d = C * (2 * l + 1)
        out[l] = x[:, idx:idx + d].reshape(x.shape[0], C, 2 * l + 1)
        idx += d
    return out


def _merge(blocks, lmax):
    return torch.cat([blocks[l].flatten(1) for l in range(lmax + 1)], dim=-1)


def _scatter_sum(x, index, n):
    out = torch.zeros((n,) + x.shape[1:], dtype=x.dtype)
    return out.index_add(0, index, x)


def _layer_norm(sd, prefix, x):
    return Fnn.layer_norm(x, (x.shape[-1],), sd[f"{prefix}.weight"], sd[f"{prefix}.bias"], 1e-5)


def main_net(sd, prefix, x, n_hidden):
    """MainNet.forward (``models/mlp.py:55-66``)."""
    x = _layer_norm(sd, f"{prefix}.input_norm", x)
    for k in range(n_hidden):
        x = Fnn.linear(x, sd[f"{prefix}.layers.{k}.weight"], sd[f"{prefix}.layers.{k}.bias"])
        x = _layer_norm(sd, f"{prefix}.layer_norms.{k}", x)
        x = Fnn.silu(x)
    return Fnn.linear(x, sd[f"{prefix}.output.weight"], sd[f"{prefix}.output.bias"])


def ictd_atom_energy(sd: Dict[str, torch.Tensor], cfg: ICTDConfig, pos, A, batch, edge_src, edge_dst,
                     edge_shifts, cell, tabs: Optional[_TPTables] = None,
                     return_features: bool = False):
    """Per-atom energy (N, 1) of PureCartesianICTDTransformerLayer.forward
    (``pure_cartesian_ictd_layers_full.py:867-1078``), no external tensor, no
    physical heads, no long-range module."""
    dtype = pos.dtype
    C, lmax, nint = cfg.channels, cfg.lmax, cfg.num_interaction
    if tabs is None:
        tabs = _TPTables(lmax, dtype, cfg.path_policy, cfg.max_rank_other)
    N = pos.shape[0]

    # edge geometry (:896-909)
    order = torch.argsort(edge_dst, stable=True)
    src, dst, shifts = edge_src[order], edge_dst[order], edge_shifts[order].to(dtype)
    shift_vec = torch.einsum("ni,nij->nj", shifts, cell[batch[src]])
    edge_vec = pos[dst] - pos[src] + shift_vec
    length = edge_vec.norm(dim=1)
    n = edge_vec / length.clamp(min=1e-8).unsqueeze(-1)
    Y = [T.direction_harmonics(n, l) for l in range(lmax + 1)]

    emb = soft_one_hot_linspace(length, 0.0, cfg.max_radius, cfg.number_of_basis,
                                basis=cfg.function_type, cutoff=True) * (cfg.number_of_basis ** 0.5)
    deg = _scatter_sum(torch.ones_like(dst), dst, N).clamp(min=1).to(dtype)

    # conv1 (:341-473)
    p = "e3_conv_emb"
    Ai = sd[f"{p}.atom_embedding.weight"][A.long()]
    Ai = _mlp(sd, f"{p}.atom_mlp", Ai, 2)
    O8 = Ai.shape[1]
    f_in = {l: Ai[src].unsqueeze(-1) * Y[l].unsqueeze(-2) for l in range(lmax + 1)}
    x2 = {l: torch.zeros(src.shape[0], O8, 2 * l + 1, dtype=dtype) for l in range(lmax + 1)}
    x2[0] = Ai[dst].unsqueeze(-1)
    gates = _mlp(sd, f"{p}.fc", emb, 3)
    blocks = harmonic_fctp(tabs, lmax, f_in, x2, sd[f"{p}.tp2.weight"], gates)
    f1 = _scatter_sum(_merge(blocks, lmax), dst, N) / deg.unsqueeze(-1)
    feats = [f1]

    # conv2..N (:938-954)
    for k in range(nint - 1):
        gates = _mlp(sd, f"fc2_layers.{k}", emb, 3)
        x1 = _split(feats[-1], C, lmax)
        x1e = {l: x1[l][src] for l in range(lmax + 1)}
        Yd = {l: Y[l].unsqueeze(-2) for l in range(lmax + 1)}
        blocks = harmonic_fctp(tabs, lmax, x1e, Yd, sd[f"tp2_layers.{k}.weight"], gates)
        feats.append(_scatter_sum(_merge(blocks, lmax), dst, N) / deg.unsqueeze(-1))

    # readout (:956-1054)
    nC = C * nint
    xb = _split(torch.cat(feats, dim=-1), nC, lmax)
    S = (nint - 1) * cfg.invariant_channels
    scalars = torch.zeros(N, S, dtype=dtype)
    for l in range(lmax + 1):
        gram = torch.einsum("ncm,ndm->ncd", xb[l], xb[l]) / ((2 * l + 1) ** 0.5)
        scalars = scalars + torch.einsum("ocd,ncd->no", sd[f"W_read.{l}"], gram)
    splits = [_split(f, C, lmax) for f in feats]
    Tb = {l: torch.cat([s[l] for s in splits], dim=-2) for l in range(lmax + 1)}
    Tb[0] = torch.cat([Tb[0], scalars.unsqueeze(-1)], dim=-2)
    p5 = []
    for l in range(lmax + 1):
        factor = T.normalized_cg(l, l, 0)[0, 0, 0].item()
        p5.append((Tb[l] * Tb[l]).sum(dim=-1) * factor)
    f_prod5 = torch.cat(p5, dim=-1)
    n_hidden = len(cfg.embed_size)
    proj = main_net(sd, "proj_total", f_prod5, n_hidden)
    e = (proj * sd["weighted_sum.weights"]).sum(dim=-1, keepdim=True)
    if return_features:
        return e, feats, f_prod5
    return e


def energy_forces_stress(sd, cfg, pos, A, batch, edge_src, edge_dst, edge_shifts, cell,
                         want_stress: bool = True, tabs=None):
    """Per-graph energy (B,), forces (N,3) = -dE/dpos, and stress (B,3,3) = (1/V) dE/d(eps)
    with the trainer's symmetric strain convention."""
    dtype = pos.dtype
    pos = pos.detach().clone().requires_grad_(True)
    nb = cell.shape[0]
    targets = [pos]
    if want_stress:
        strain = torch.zeros(nb, 3, 3, dtype=dtype, requires_grad=True)
        D = torch.eye(3, dtype=dtype) + 0.5 * (strain + strain.transpose(-1, -2))
        pos_in = torch.einsum("ni,nij->nj", pos, D[batch])
        cell_in = torch.bmm(cell.to(dtype), D)
        targets.append(strain)
    else:
        pos_in, cell_in = pos, cell.to(dtype)
    e = ictd_atom_energy(sd, cfg, pos_in, A, batch, edge_src, edge_dst, edge_shifts, cell_in, tabs=tabs)
    Eg = _scatter_sum(e.squeeze(-1), batch, nb)
    grads = torch.autograd.grad(Eg.sum(), targets)
    F = -grads[0]
    out = {"energy": Eg.detach(), "forces": F.detach(), "atom_energy": e.detach().squeeze(-1)}
    if want_stress:
        vol = torch.abs(torch.det(cell.to(dtype))).clamp(min=1e-10)
        out["stress"] = (grads[1] / vol.view(-1, 1, 1)).detach()
    return out
