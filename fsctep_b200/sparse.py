"""pure-cartesian-sparse on B200: weight packing and the native E + F engine.

Host-side mirror of ``PureCartesianSparseTransformerLayer``
(``models/pure_cartesian_sparse_layers.py:459-855``) with the options its configurations use
(``max_rank_other=1``, ``k_policy="k0"``): ``SparseEngine`` packs a reference-layout
``state_dict`` into the device layouts of ``fsc_sparse_weights`` (include/fsctep_b200.h) and runs
``fsc_sparse_forward`` / ``fsc_sparse_backward``.  The packing is a one-time weight transform:
per-species-pair conv1 tables (fc.4 contracted with the atom features of both edge ends) and the
conv2 fc.4 weights regrouped per output rank for the after-aggregation GEMMs.
"""

from __future__ import annotations

import ctypes as C
import math
from dataclasses import dataclass, field
from typing import Dict, List, Sequence, Tuple

import torch

from fsctep_b200 import _native as N
from fsctep_b200.ictd import BASIS_KINDS, GraphCSR

J = 65  # radial hidden width + bias row


def sparse_paths(lmax: int) -> List[Tuple[int, int, int]]:
    """(L1, L2, Lout) of PureCartesianTensorProductO3Sparse with max_rank_other=1, k0, no epsilon,
    in the reference order (``pure_cartesian.py:353-418``)."""
    return [(L1, L2, L1 + L2) for L1 in range(lmax + 1) for L2 in range(lmax + 1)
            if min(L1, L2) <= 1 and L1 + L2 <= lmax]


@dataclass
class SparseConfig:
    channels: int = 64
    lmax: int = 2
    num_interaction: int = 3
    number_of_basis: int = 8
    max_radius: float = 5.0
    function_type: str = "gaussian"
    output_size: int = 8
    embedding_dim: int = 16
    max_atomvalue: int = 10
    invariant_channels: int = 32
    embed_size: Sequence[int] = field(default_factory=lambda: (128, 128, 128))

    def native(self) -> N.SparseConfig:
        if self.function_type not in BASIS_KINDS:
            raise NotImplementedError(f"radial basis {self.function_type!r} is not implemented")
        if self.output_size != 8:
            raise NotImplementedError("pure-cartesian-sparse engine: output_size must be 8")
        c = N.SparseConfig(channels=self.channels, lmax=self.lmax, num_interaction=self.num_interaction,
                           number_of_basis=self.number_of_basis, basis_kind=BASIS_KINDS[self.function_type],
                           max_radius=float(self.max_radius), num_species=self.max_atomvalue,
                           invariant_channels=self.invariant_channels, n_hidden=len(self.embed_size), n_out=17)
        for k, h in enumerate(self.embed_size):
            c.hidden[k] = int(h)
        return c


def _silu(x):
    return x * torch.sigmoid(x)


class PackedSparseWeights:
    """fp32 device tensors in the fsc_sparse_weights layouts, from a reference state_dict."""

    def __init__(self, sd: Dict[str, torch.Tensor], cfg: SparseConfig, device):
        dev = torch.device(device)
        f64 = lambda k: sd[k].detach().to(device=dev, dtype=torch.float64)  # noqa: E731
        C_, L, nint = cfg.channels, cfg.lmax, cfg.num_interaction
        paths = sparse_paths(L)
        P = len(paths)
        keep = {}

        def put(name, t):
            keep[name] = t.to(device=dev, dtype=torch.float32).contiguous()

        # radial MLP hidden layers: conv1 (e3_conv_emb.fc), then e3_conv_layers.k.fc
        pref = ["e3_conv_emb.fc"] + [f"e3_conv_layers.{k}.fc" for k in range(1, nint)]
        put("rad_w1", torch.stack([f64(f"{p}.0.weight") for p in pref]))
        put("rad_b1", torch.stack([f64(f"{p}.0.bias") for p in pref]))
        put("rad_w2", torch.stack([f64(f"{p}.2.weight") for p in pref]))
        put("rad_b2", torch.stack([f64(f"{p}.2.bias") for p in pref]))

        # conv1: K[ss][sd][L][j][c] = sum_{a,b} W[(p_L, c, a, b), j] ai[ss][a] ai[sd][b]
        emb = f64("e3_conv_emb.atom_embedding.weight")
        h = _silu(emb @ f64("e3_conv_emb.atom_mlp.0.weight").T + f64("e3_conv_emb.atom_mlp.0.bias"))
        ai = h @ f64("e3_conv_emb.atom_mlp.2.weight").T + f64("e3_conv_emb.atom_mlp.2.bias")  # [S, 8]
        O8 = ai.shape[1]
        W4 = torch.cat([f64("e3_conv_emb.fc.4.weight"), f64("e3_conv_emb.fc.4.bias")[:, None]], dim=1)  # [P*C*64, J]
        W4 = W4.reshape(P, C_, O8, O8, J)
        Ks = []
        for Lr in range(L + 1):
            p = paths.index((Lr, 0, Lr))
            Ks.append(torch.einsum("cabj,sa,tb->stjc", W4[p], ai, ai))
        put("pair_k", torch.stack(Ks, dim=2))  # [S, S, L+1, J, C]

        # conv2: per layer and output rank, blocks [(q, j, a)][c] and their transposes
        mix, mixT = [], []
        for k in range(1, nint):
            Wk = torch.cat([f64(f"e3_conv_layers.{k}.fc.4.weight"), f64(f"e3_conv_layers.{k}.fc.4.bias")[:, None]],
                           dim=1).reshape(P, C_, C_, J)  # [p, c, a, j]
            for Lo in range(L + 1):
                ps = [i for i, pth in enumerate(paths) if pth[2] == Lo]
                blk = torch.stack([Wk[p].permute(2, 1, 0) for p in ps])  # [q, j, a, c]
                blk = blk.reshape(len(ps) * J * C_, C_)
                mix.append(blk.reshape(-1))
                mixT.append(blk.T.contiguous().reshape(-1))
        put("mix", torch.cat(mix))
        put("mixT", torch.cat(mixT))

        # readout bilinear invariants (product_3.W.L / sqrt(3^L)), packed upper triangle
        nC = C_ * nint
        iu = torch.triu_indices(nC, nC, device=dev)
        wp, ws = [], []
        for Lr in range(L + 1):
            Wr = f64(f"product_3.W.{Lr}") / math.sqrt(3 ** Lr)
            ws.append((0.5 * (Wr + Wr.transpose(1, 2))).reshape(-1))
            packed = (Wr + Wr.transpose(1, 2))[:, iu[0], iu[1]]
            diag = iu[0] == iu[1]
            packed[:, diag] = Wr[:, iu[0][diag], iu[1][diag]]
            wp.append(packed.reshape(-1))
        put("wread_p", torch.cat(wp))
        put("wread_s", torch.cat(ws))
        keep["pairs"] = (iu[0] | (iu[1] << 16)).to(torch.int32).contiguous()

        put("mn_in_g", f64("proj_total.input_norm.weight"))
        put("mn_in_b", f64("proj_total.input_norm.bias"))
        for k in range(len(cfg.embed_size)):
            put(f"mn_w{k}", f64(f"proj_total.layers.{k}.weight"))
            put(f"mn_b{k}", f64(f"proj_total.layers.{k}.bias"))
            put(f"mn_g{k}", f64(f"proj_total.layer_norms.{k}.weight"))
            put(f"mn_beta{k}", f64(f"proj_total.layer_norms.{k}.bias"))
        wsum = f64("weighted_sum.weights")
        put("out_v", f64("proj_total.output.weight").T @ wsum)
        self.out_c0 = float((f64("proj_total.output.bias") * wsum).sum().item())
        self.tensors = keep
        s = N.SparseWeights()
        for name in ("rad_w1", "rad_b1", "rad_w2", "rad_b2", "pair_k", "mix", "mixT", "wread_p", "wread_s", "pairs",
                     "mn_in_g", "mn_in_b", "out_v"):
            setattr(s, name, keep[name].data_ptr())
        for k in range(len(cfg.embed_size)):
            s.mn_w[k] = keep[f"mn_w{k}"].data_ptr()
            s.mn_b[k] = keep[f"mn_b{k}"].data_ptr()
            s.mn_g[k] = keep[f"mn_g{k}"].data_ptr()
            s.mn_beta[k] = keep[f"mn_beta{k}"].data_ptr()
        s.out_c0 = self.out_c0
        self.struct = s


class SparseEngine:
    """Native energy + forces of one packed pure-cartesian-sparse model."""

    def __init__(self, state_dict: Dict[str, torch.Tensor], cfg: SparseConfig, device="cuda"):
        self.cfg = cfg
        self.device = torch.device(device)
        self.ncfg = cfg.native()
        self.weights = PackedSparseWeights(state_dict, cfg, self.device)
        self._ws = None

    def workspace(self, num_atoms: int, num_edges: int):
        need = N.lib().fsc_sparse_workspace_bytes(C.byref(self.ncfg), num_atoms, num_edges)
        if need == 0:
            N.check(1, "fsc_sparse_workspace_bytes (unsupported configuration)")
        if self._ws is None or self._ws.numel() < need:
            self._ws = None
            self._ws = torch.empty(need, dtype=torch.uint8, device=self.device)
        return self._ws

    def _graph(self, pos, species, batch, cell, g: GraphCSR, num_graphs, num_local, energy_weight):
        s = N.Graph()
        s.num_atoms = g.num_atoms
        s.num_local = g.num_atoms if num_local is None else int(num_local)
        s.num_edges = g.num_edges
        s.num_graphs = int(num_graphs)
        s.pos, s.species, s.batch, s.cell = pos.data_ptr(), species.data_ptr(), batch.data_ptr(), cell.data_ptr()
        s.row_ptr, s.src, s.shift = g.row_ptr.data_ptr(), g.src.data_ptr(), g.shift.data_ptr()
        s.tr_ptr, s.tr_eid = g.tr_ptr.data_ptr(), g.tr_eid.data_ptr()
        s.energy_weight = 0 if energy_weight is None else energy_weight.data_ptr()
        s.field = 0
        return s

    def forward(self, pos, species, batch, cell, g: GraphCSR, num_local=None, avg_num_neighbors=None):
        """``avg_num_neighbors``: the conv2 normaliser; None = E / N of this graph (the reference's
        per-call value).  The backward of this forward uses the same value."""
        self.ncfg.avg_num_neighbors = 0.0 if avg_num_neighbors is None else float(avg_num_neighbors)
        pos = pos.detach().to(torch.float32).contiguous()
        species = species.to(torch.int32).contiguous()
        batch = batch.to(torch.int32).contiguous()
        cell = cell.detach().to(torch.float32).reshape(-1, 3, 3).contiguous()
        B = cell.shape[0]
        ws = self.workspace(g.num_atoms, g.num_edges)
        energy = torch.empty(B, dtype=torch.float32, device=self.device)
        atom_e = torch.empty(g.num_atoms, dtype=torch.float32, device=self.device)
        gs = self._graph(pos, species, batch, cell, g, B, num_local, None)
        N.check(N.lib().fsc_sparse_forward(C.byref(self.ncfg), C.byref(self.weights.struct), C.byref(gs),
                                           N.ptr(energy), N.ptr(atom_e), N.ptr(ws), ws.numel(),
                                           N.stream_ptr(self.device)), "fsc_sparse_forward")
        self._last = (pos, species, batch, cell, g, num_local)
        return energy, atom_e

    def backward(self, energy_weight=None, want_virial=True, want_cell_grad=False, want_edge_grad=False):
        pos, species, batch, cell, g, num_local = self._last
        B = cell.shape[0]
        ws = self.workspace(g.num_atoms, g.num_edges)
        dev = self.device
        out = {"forces": torch.empty(g.num_atoms, 3, dtype=torch.float32, device=dev)}
        if want_virial:
            out["virial"] = torch.empty(B, 3, 3, dtype=torch.float32, device=dev)
        if want_cell_grad:
            out["cell_grad"] = torch.empty(B, 3, 3, dtype=torch.float32, device=dev)
        if want_edge_grad:
            out["edge_grad"] = torch.empty(g.num_edges, 3, dtype=torch.float32, device=dev)
        if energy_weight is not None:
            energy_weight = energy_weight.detach().to(torch.float32).reshape(-1).contiguous()
        gs = self._graph(pos, species, batch, cell, g, B, num_local, energy_weight)
        o = N.IctdOutputs()
        o.forces = out["forces"].data_ptr()
        o.virial = out["virial"].data_ptr() if want_virial else 0
        o.cell_grad = out["cell_grad"].data_ptr() if want_cell_grad else 0
        o.edge_grad = out["edge_grad"].data_ptr() if want_edge_grad else 0
        N.check(N.lib().fsc_sparse_backward(C.byref(self.ncfg), C.byref(self.weights.struct), C.byref(gs),
                                            C.byref(o), N.ptr(ws), ws.numel(), N.stream_ptr(dev)), "fsc_sparse_backward")
        return out

    # ---- stepwise evaluation (per-layer ghost-feature exchange of a decomposition)
    def _rows(self):
        return sum(3 ** L for L in range(self.cfg.lmax + 1))

    def feature_buffer(self, which: int, layer: int):
        """View (num_atoms, R, C) of layer ``layer``'s features (which = 0) or their gradient
        (which = 1) in the workspace of the last call."""
        g = self._last[4]
        ws = self.workspace(g.num_atoms, g.num_edges)
        addr = C.c_void_p(0)
        N.check(N.lib().fsc_sparse_feature_buffer(C.byref(self.ncfg), g.num_atoms, g.num_edges, N.ptr(ws), which,
                                                  layer, C.byref(addr)), "fsc_sparse_feature_buffer")
        off = int(addr.value) - ws.data_ptr()
        R, Cc = self._rows(), self.cfg.channels
        return ws[off:off + g.num_atoms * R * Cc * 4].view(torch.float32).view(g.num_atoms, R, Cc)

    def begin_steps(self, pos, species, batch, cell, g: GraphCSR, num_local=None, avg_num_neighbors=None,
                    layer_atoms=None):
        if layer_atoms is not None:
            raise ValueError("the sparse engine evaluates every layer on all atoms (no layer_atoms)")
        self.ncfg.avg_num_neighbors = 0.0 if avg_num_neighbors is None else float(avg_num_neighbors)
        pos = pos.detach().to(torch.float32).contiguous()
        species = species.to(torch.int32).contiguous()
        batch = batch.to(torch.int32).contiguous()
        cell = cell.detach().to(torch.float32).reshape(-1, 3, 3).contiguous()
        self.workspace(g.num_atoms, g.num_edges)
        self._last = (pos, species, batch, cell, g, num_local)
        self._step_out = (torch.empty(cell.shape[0], dtype=torch.float32, device=self.device),
                          torch.empty(g.num_atoms, dtype=torch.float32, device=self.device))

    def forward_step(self, step: int):
        pos, species, batch, cell, g, num_local = self._last
        ws = self.workspace(g.num_atoms, g.num_edges)
        energy, atom_e = self._step_out
        gs = self._graph(pos, species, batch, cell, g, cell.shape[0], num_local, None)
        last = step == self.cfg.num_interaction
        N.check(N.lib().fsc_sparse_forward_step(C.byref(self.ncfg), C.byref(self.weights.struct), C.byref(gs), step,
                                                N.ptr(energy) if last else None, N.ptr(atom_e) if last else None,
                                                N.ptr(ws), ws.numel(), N.stream_ptr(self.device)),
                f"fsc_sparse_forward_step({step})")
        return (energy, atom_e) if last else self.feature_buffer(0, step)

    def begin_backward(self, energy_weight=None, want_virial=True, want_cell_grad=False, want_edge_grad=False):
        g, B = self._last[4], self._last[3].shape[0]
        dev = self.device
        out = {"forces": torch.empty(g.num_atoms, 3, dtype=torch.float32, device=dev)}
        if want_virial:
            out["virial"] = torch.empty(B, 3, 3, dtype=torch.float32, device=dev)
        if want_cell_grad:
            out["cell_grad"] = torch.empty(B, 3, 3, dtype=torch.float32, device=dev)
        if want_edge_grad:
            out["edge_grad"] = torch.empty(g.num_edges, 3, dtype=torch.float32, device=dev)
        o = N.IctdOutputs()
        o.forces = out["forces"].data_ptr()
        o.virial = out["virial"].data_ptr() if want_virial else 0
        o.cell_grad = out["cell_grad"].data_ptr() if want_cell_grad else 0
        o.edge_grad = out["edge_grad"].data_ptr() if want_edge_grad else 0
        if energy_weight is not None:
            energy_weight = energy_weight.detach().to(torch.float32).reshape(-1).contiguous()
        self._bwd = (out, o, energy_weight)
        return out

    def backward_step(self, step: int):
        pos, species, batch, cell, g, num_local = self._last
        ws = self.workspace(g.num_atoms, g.num_edges)
        out, o, ew = self._bwd
        gs = self._graph(pos, species, batch, cell, g, cell.shape[0], num_local, ew)
        N.check(N.lib().fsc_sparse_backward_step(C.byref(self.ncfg), C.byref(self.weights.struct), C.byref(gs),
                                                 step, C.byref(o), N.ptr(ws), ws.numel(), N.stream_ptr(self.device)),
                f"fsc_sparse_backward_step({step})")
        return self.feature_buffer(1, step - 1) if step >= 1 else out

    def status(self) -> int:
        pos, species, batch, cell, g, num_local = self._last
        ws = self.workspace(g.num_atoms, g.num_edges)
        st = C.c_int(0)
        N.check(N.lib().fsc_sparse_status(C.byref(self.ncfg), g.num_atoms, g.num_edges, N.ptr(ws),
                                          N.stream_ptr(self.device), C.byref(st)), "fsc_sparse_status")
        return int(st.value)

    def energy_forces(self, pos, species, batch, cell, g: GraphCSR, num_local=None, want_stress=True):
        energy, atom_e = self.forward(pos, species, batch, cell, g, num_local)
        out = self.backward(want_virial=want_stress)
        out["energy"] = energy
        out["atom_energy"] = atom_e
        if want_stress:
            vol = torch.abs(torch.det(self._last[3].double())).clamp(min=1e-10).float()
            v = out["virial"]
            out["stress"] = 0.5 * (v + v.transpose(1, 2)) / vol.view(-1, 1, 1)
        return out


# Field order of the core.pt weight blob of fsctep::sparse_atom_energy (torch_ops/ictd_op.cpp).
SPARSE_BLOB_FIELDS = (["rad_w1", "rad_b1", "rad_w2", "rad_b2", "pair_k", "mix", "mixT", "wread_p", "wread_s", "pairs",
                       "mn_in_g", "mn_in_b"] + [f"mn_w{k}" for k in range(4)] + [f"mn_b{k}" for k in range(4)]
                      + [f"mn_g{k}" for k in range(4)] + [f"mn_beta{k}" for k in range(4)] + ["out_v"])


def sparse_weight_blob(packed: "PackedSparseWeights", cfg: SparseConfig):
    """One float32 device tensor holding every packed sparse weight array (int32 arrays
    bit-cast), each field 256-byte aligned, plus the integer / float configuration lists of the
    core.pt op."""
    parts, offs, cur = [], [], 0
    for name in SPARSE_BLOB_FIELDS:
        t = packed.tensors.get(name)
        if t is None:
            offs.append(-1)
            continue
        flat = t.reshape(-1)
        flat = flat.view(torch.float32) if flat.dtype == torch.int32 else flat.to(torch.float32)
        pad = (-cur) % 64
        if pad:
            parts.append(torch.zeros(pad, dtype=torch.float32, device=flat.device))
            cur += pad
        offs.append(cur)
        parts.append(flat)
        cur += flat.numel()
    blob = torch.cat(parts).contiguous()
    nc = cfg.native()
    icfg = [nc.channels, nc.lmax, nc.num_interaction, nc.number_of_basis, nc.basis_kind, nc.num_species,
            nc.invariant_channels, nc.n_hidden] + [int(nc.hidden[k]) for k in range(4)] + [nc.n_out] + offs
    fcfg = [float(cfg.max_radius), float(packed.out_c0)]
    return blob, icfg, fcfg
