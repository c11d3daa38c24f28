"""pure-cartesian-ictd on B200: weight packing, graph CSR and the native E + F engine.

Host-side mirror of the reference operator surface for this path:

* ``ICTDEngine`` packs a reference-layout ``state_dict`` of
  ``PureCartesianICTDTransformerLayer`` (``models/pure_cartesian_ictd_layers_full.py``)
  into the fp32 device layouts of ``include/fsctep_b200.h`` and runs the native
  forward / hand-written backward (``fsc_ictd_forward`` / ``fsc_ictd_backward``).
* ``GraphCSR`` turns an edge list ``(edge_src, edge_dst, edge_shifts)`` (any order) into
  the dst-sorted CSR + transpose CSR the kernels read.
* ``PureCartesianICTDTransformerLayer`` (in ``fsctep_b200.models``) wraps both behind the
  reference module's constructor, state_dict keys and ``forward`` signature.

Nothing here computes on the CPU: every numeric step of the path is a kernel in
``libfsctep_b200.so``; the packing below is a one-time weight transform.
"""

from __future__ import annotations

import ctypes as C
import math
from dataclasses import dataclass, field
from typing import Dict, Optional, Sequence

import torch

from fsctep_b200 import _native as N
from fsctep_b200 import tables as T

BASIS_KINDS = {"gaussian": 0, "bessel": 1}
NP = 11
P3_PATHS = [[0, 4, 9], [1, 3, 6, 8], [2, 5, 7, 10]]   # paths by l3, path order
P1_PATHS = [[0, 1, 2], [3, 4, 5, 6], [7, 8, 9, 10]]   # paths by l1
P_L0L = [0, 3, 7]                                      # (l,0,l) paths
# pure-cartesian-ictd-o3 (active irreps 0e, 1e, 1o, 2e; pure_cartesian_ictd_layers_o3.py): index in
# its 17-path list (ictd_irreps.py:1356-1366) of each SO(3) path above, carried by the
# canonical-parity blocks 0e, 1o, 2e.  The 1e block only couples to itself and starts at zero.
# With active irreps 0e,1o,2e (the "auto" preset) the o3 path list is the SO(3) one, in order.
SO3_TO_O3 = [0, 2, 3, 8, 9, 10, 11, 12, 14, 15, 16]


def o3_num_paths(irreps) -> int:
    return 17 if "1e" in irreps else 11


@dataclass
class ICTDConfig:
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
    o3: bool = False  # pure-cartesian-ictd-o3 (parity-keyed irreps, external field, tensor heads)
    o3_irreps: Sequence[str] = ("0e", "1e", "1o", "2e")  # active irreps of the o3 model

    @property
    def scalar_channels(self):
        return (self.num_interaction - 1) * self.invariant_channels

    def native(self) -> N.IctdConfig:
        if self.function_type not in BASIS_KINDS:
            raise NotImplementedError(f"radial basis {self.function_type!r} is not implemented in the sm_100a kernels "
                                      f"(supported: {sorted(BASIS_KINDS)})")
        c = N.IctdConfig(channels=self.channels, lmax=self.lmax, num_interaction=self.num_interaction,
                         number_of_basis=self.number_of_basis, basis_kind=BASIS_KINDS[self.function_type],
                         max_radius=float(self.max_radius), num_species=self.max_atomvalue,
                         output_size=self.output_size, invariant_channels=self.invariant_channels,
                         n_hidden=len(self.embed_size), n_out=17,
                         o3=1 if (self.o3 and "1e" in self.o3_irreps) else 0)
        for k, h in enumerate(self.embed_size):
            c.hidden[k] = int(h)
        return c


def gram_xmap(C: int, nint: int, o3: bool = False):
    """Storage location of every element of the readout's Gram operand.

    The reference splits the flat concatenation of all layers' features into blocks of
    nC*(2l+1) elements (``pure_cartesian_ictd_layers_full.py:956-958``; the o3 model the same way
    over its 0e,1e,1o,2e blocks, ``pure_cartesian_ictd_layers_o3.py:976``), so element m of
    channel c of block b is flat element off_b + c*(2l_b+1) + m, with each layer's features
    laid out [l0 (C,1) | l1 (C,3) | l2 (C,5)] (o3: [0e | 1e | 1o | 2e]).  Returns, per flat
    element, (layer << 16) | (k*C + channel) with k = l*l + m the component index in the
    [N][9][C] feature buffers, or -1 for the o3 model's 1e block (identically zero, no storage).
    """
    if o3:
        blocks = [(0, 0), (None, 1), (1, 1), (2, 2)]  # (storage l or None, l) per block
    else:
        blocks = [(0, 0), (1, 1), (2, 2)]
    per_layer = sum(C * (2 * l + 1) for _, l in blocks)
    out = []
    for q in range(per_layer * nint):
        layer, w = divmod(q, per_layer)
        base = 0
        for sl, l in blocks:
            width = C * (2 * l + 1)
            if w < base + width:
                break
            base += width
        c, m = divmod(w - base, 2 * l + 1)
        out.append(-1 if sl is None else (layer << 16) | ((sl * sl + m) * C + c))
    return out


def gram_xinv(C: int, nint: int, o3: bool = False):
    """Inverse of gram_xmap: [nint][9*C] storage (layer, k*C + c) -> Gram operand row."""
    inv = [[0] * (9 * C) for _ in range(nint)]
    for r, code in enumerate(gram_xmap(C, nint, o3)):
        if code >= 0:
            inv[code >> 16][code & 0xFFFF] = r
    return inv


def f16_image(x: torch.Tensor) -> torch.Tensor:
    """float64 operand image [blocks][...] -> float32 tensor holding a 64-byte header (element 0 =
    1/scale) and, per block, the fp16 hi plane then the fp16 lo plane of scale * x, where scale is
    the power of two that brings max |x| to at most 2^14 (hi = fp16(x s), lo = fp16(x s - hi))."""
    m = float(x.abs().max().item()) if x.numel() else 0.0
    scale = 2.0 ** (14 - math.ceil(math.log2(m))) if m > 0 else 1.0
    xs = x * scale
    hi = xs.to(torch.float16)
    lo = (xs - hi.to(torch.float64)).to(torch.float16)
    planes = torch.stack([hi, lo], dim=1).reshape(-1).contiguous()
    header = torch.zeros(16, dtype=torch.float32, device=x.device)
    header[0] = 1.0 / scale
    return torch.cat([header, planes.view(torch.float32)])


def readout_images(W_read, C: int, nint: int, ls=(0, 1, 2)):
    """W_read blocks (Gram block b has l = ls[b]) as shared-memory images of the tcgen05 kind::f16
    operands (see include/fsctep_b200.h).  Returns (wimg_fwd, wimg_bwd), each a header + fp16 planes
    (:func:`f16_image`) in a float32 tensor.
    """
    nC = C * nint
    nb = nC // 8
    fwd, bwd = [], []
    iu = torch.triu_indices(nb, nb)
    for W_b, l in zip(W_read, ls):
        Wr = W_b.to(torch.float64) / math.sqrt(2 * l + 1)
        S = Wr.shape[0]
        Ws = 0.5 * (Wr + Wr.transpose(1, 2))
        blk = Ws.reshape(S, nb, 8, nb, 8).permute(1, 3, 0, 2, 4).reshape(nb, nb, S, 64)  # [cb][db][o][pair]
        # forward: cb <= db, x2 off the diagonal, pairs reordered (c = 4ch + ci, d = 4dh + di) ->
        # 16qq + 4ci + di with qq = ch + 2dh (the generator thread of quarter qq owns those c and d
        # rows); B = [k/8][o][k%8], K = pairs
        f = blk[iu[0], iu[1]] * torch.where(iu[0] == iu[1], 1.0, 2.0).to(blk)[:, None, None]
        f = f.reshape(-1, S, 2, 4, 2, 4).permute(0, 1, 4, 2, 3, 5).reshape(-1, S, 64)
        fwd.append(f.reshape(-1, S, 8, 8).permute(0, 2, 1, 3))
        # backward: all blocks in pairs of d-blocks (db even, db + 1) -> N = 128 pairs per MMA,
        # B = [o/8][pair of the two blocks][o%8], K = outputs o; within a block the pairs are
        # ordered (c/4, d, c%4): epilogue quarter (d-block of the pair, c/4) reads its 32 columns
        # at once, c-rows c, c + 1 side by side
        bo = blk.reshape(nb, nb, S, 2, 4, 8).permute(0, 1, 2, 3, 5, 4).reshape(nb, nb, S, 64)
        b = bo.reshape(nb, nb // 2, 2, S, 64).permute(0, 1, 3, 2, 4).reshape(nb * nb // 2, S, 128)
        bwd.append(b.reshape(-1, S // 8, 8, 128).permute(0, 1, 3, 2))
    return f16_image(torch.cat(fwd)), f16_image(torch.cat(bwd))


def _silu(x):
    return x * torch.sigmoid(x)


class PackedICTDWeights:
    """fp32 device tensors in the C-ABI layouts, derived once from a reference state_dict."""

    def __init__(self, sd: Dict[str, torch.Tensor], cfg: ICTDConfig, device):
        dev = torch.device(device)
        f64 = lambda k: sd[k].detach().to(device=dev, dtype=torch.float64)  # noqa: E731
        C_, nint = cfg.channels, cfg.num_interaction
        keep = {}

        def put(name, t):
            keep[name] = t.to(device=dev, dtype=torch.float32).contiguous()
            return keep[name]

        o3 = bool(cfg.o3)
        irreps = tuple(cfg.o3_irreps) if o3 else ()
        four = "1e" in irreps  # 0e,1e,1o,2e: 17 paths, the SO(3) path p is o3 path SO3_TO_O3[p]
        psel = (lambda t: t[SO3_TO_O3]) if four else (lambda t: t)  # noqa: E731
        put("tables", torch.from_numpy(T.kernel_tables(cfg.lmax)))
        # per-species conv1 tables
        emb = f64("e3_conv_emb.atom_embedding.weight")
        h = _silu(emb @ f64("e3_conv_emb.atom_mlp.0.weight").T + f64("e3_conv_emb.atom_mlp.0.bias"))
        ai = h @ f64("e3_conv_emb.atom_mlp.2.weight").T + f64("e3_conv_emb.atom_mlp.2.bias")  # [S, 8]
        W1 = psel(f64("e3_conv_emb.tp2.weight"))  # [P, C, 8, 8]
        vsp = torch.stack([torch.einsum("oij,sj->sio", W1[p], ai) for p in P_L0L], dim=1)  # [S, 3, 8, C]
        put("ai", ai)
        put("vsp", vsp)
        # radial MLPs: conv1 fc, then fc2_layers.k
        pref = ["e3_conv_emb.fc"] + [f"fc2_layers.{k}" for k in range(nint - 1)]
        put("rad_w1", torch.stack([f64(f"{p}.0.weight") for p in pref]))
        put("rad_b1", torch.stack([f64(f"{p}.0.bias") for p in pref]))
        put("rad_w2", torch.stack([f64(f"{p}.2.weight") for p in pref]))
        put("rad_b2", torch.stack([f64(f"{p}.2.bias") for p in pref]))
        put("rad_w3", torch.stack([psel(f64(f"{p}.4.weight")) for p in pref]))
        put("rad_b3", torch.stack([psel(f64(f"{p}.4.bias")) for p in pref]))
        # channel mixes
        fwd, bwd, dx = [], [], []
        for k in range(nint - 1):
            W = psel(f64(f"tp2_layers.{k}.weight"))[..., 0]  # [P, o, i]
            for group in P3_PATHS:
                fwd.append(torch.cat([W[p].T for p in group], dim=0).reshape(-1))      # [(rank,i)][o]
                bwd.append(torch.cat([W[p] for p in group], dim=1).reshape(-1))        # [o][(rank,i)]
            for group in P1_PATHS:
                dx.append(torch.cat([W[p] for p in group], dim=0).reshape(-1))         # [(rank,o)][i]
        put("mix_fwd", torch.cat(fwd))
        put("mix_bwd", torch.cat(bwd))
        put("mix_dx", torch.cat(dx))
        # readout W_read, one block per Gram block (l = 0, 1, 2; o3: 0e, 1e, 1o, 2e)
        nC = C_ * nint
        if o3:
            wkeys, ls = [f"W_read.{k}" for k in irreps], [int(k[0]) for k in irreps]
        else:
            wkeys, ls = [f"W_read.{l}" for l in range(3)], [0, 1, 2]
        iu = torch.triu_indices(nC, nC, device=dev)
        wp, ws = [], []
        for key, l in zip(wkeys, ls):
            Wr = f64(key) / math.sqrt(2 * l + 1)  # [S, nC, nC]
            Wsym = 0.5 * (Wr + Wr.transpose(1, 2))
            ws.append(Wsym.reshape(-1))
            packed = (Wr + Wr.transpose(1, 2))[:, iu[0], iu[1]]
            diag = iu[0] == iu[1]
            packed[:, diag] = Wr[:, iu[0][diag], iu[1][diag]]
            wp.append(packed.reshape(-1))
        put("wread_p", torch.cat(wp))
        put("wread_s", torch.cat(ws))
        keep["pairs"] = (iu[0] | (iu[1] << 16)).to(torch.int32).contiguous()
        keep["xmap"] = torch.tensor(gram_xmap(C_, nint, four), dtype=torch.int32, device=dev)
        keep["xinv"] = torch.tensor(gram_xinv(C_, nint, four), dtype=torch.int32, device=dev).reshape(-1)
        S = (nint - 1) * cfg.invariant_channels
        if S in (32, 64) and nC % 8 == 0:
            wf, wb = readout_images([f64(k) for k in wkeys], C_, nint, ls)
            put("wimg_fwd", wf)
            put("wimg_bwd", wb)
        else:
            keep["wimg_fwd"] = keep["wimg_bwd"] = None
        # o3: external-field scale of the 1o block and the physical-tensor heads (canonical parity
        # of each head's l), in state_dict order
        skey = "e3_conv_emb.external_tensor_scale_by_irrep"
        self.field_scale = float(sd[skey][irreps.index("1o")]) if o3 and skey in sd else 0.0
        self.heads = []  # (name, l, Gram block)
        hw = []
        for key in sd:
            parts = key.split(".")
            if o3 and len(parts) == 4 and parts[0] == "physical_tensor_heads" and parts[3] == "weight":
                l = int(parts[2])
                self.heads.append((parts[1], l, irreps.index(f"{l}{'e' if l % 2 == 0 else 'o'}")))
                hw.append(f64(key).reshape(-1))
        keep["heads_w"] = torch.stack(hw).to(torch.float32).contiguous() if hw else None
        # MainNet
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
        s = N.IctdWeights()
        for name in ("tables", "ai", "vsp", "rad_w1", "rad_b1", "rad_w2", "rad_b2", "rad_w3", "rad_b3",
                     "mix_fwd", "mix_bwd", "mix_dx", "wread_p", "wread_s", "pairs", "xmap", "xinv", "mn_in_g", "mn_in_b", "out_v"):
            setattr(s, name, keep[name].data_ptr())
        for k in range(len(cfg.embed_size)):
            s.mn_w[k] = keep[f"mn_w{k}"].data_ptr()
            s.mn_b[k] = keep[f"mn_b{k}"].data_ptr()
            s.mn_g[k] = keep[f"mn_g{k}"].data_ptr()
            s.mn_beta[k] = keep[f"mn_beta{k}"].data_ptr()
        s.out_c0 = self.out_c0
        s.wimg_fwd = 0 if keep["wimg_fwd"] is None else keep["wimg_fwd"].data_ptr()
        s.wimg_bwd = 0 if keep["wimg_bwd"] is None else keep["wimg_bwd"].data_ptr()
        self.struct = s


# Field order of the core.pt weight blob (fsctep::ictd_atom_energy, torch_ops/ictd_op.cpp).
BLOB_FIELDS = (["tables", "ai", "vsp", "rad_w1", "rad_b1", "rad_w2", "rad_b2", "rad_w3", "rad_b3", "mix_fwd",
                "mix_bwd", "mix_dx", "wread_p", "wread_s", "pairs", "xmap", "xinv", "wimg_fwd", "wimg_bwd",
                "mn_in_g", "mn_in_b"] + [f"mn_w{k}" for k in range(4)] + [f"mn_b{k}" for k in range(4)]
               + [f"mn_g{k}" for k in range(4)] + [f"mn_beta{k}" for k in range(4)] + ["out_v"])


def weight_blob(packed: "PackedICTDWeights", cfg: "ICTDConfig"):
    """One float32 device tensor holding every packed weight array (int32 arrays bit-cast), each
    field 256-byte aligned, plus the integer / float configuration lists of the core.pt op."""
    parts, offs, cur = [], [], 0
    for name in BLOB_FIELDS:
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
            nc.output_size, nc.invariant_channels, nc.n_hidden] + [int(nc.hidden[k]) for k in range(4)] + \
           [nc.n_out, nc.o3] + offs
    fcfg = [float(cfg.max_radius), float(packed.out_c0)]
    return blob, icfg, fcfg


class GraphCSR:
    """dst-sorted CSR + transpose CSR of an edge list (all int32 on the device).

    ``order`` maps CSR edge slots to the caller's edge indices (stable by dst), so per-edge
    outputs can be returned in the caller's order.
    """

    def __init__(self, num_atoms: int, row_ptr, src, shift, tr_ptr, tr_eid, order=None):
        self.num_atoms = int(num_atoms)
        self.row_ptr, self.src, self.shift, self.tr_ptr, self.tr_eid = row_ptr, src, shift, tr_ptr, tr_eid
        self.order = order
        self.num_edges = int(src.shape[0])

    @staticmethod
    def transpose(row_ptr, src, num_atoms: int):
        dev = src.device
        E = int(src.shape[0])
        tr_ptr = torch.empty(num_atoms + 1, dtype=torch.int32, device=dev)
        tr_eid = torch.empty(max(E, 1), dtype=torch.int32, device=dev)
        L = N.lib()
        ws_bytes = L.fsc_csr_transpose_workspace_bytes(num_atoms, E)
        ws = torch.empty(ws_bytes, dtype=torch.uint8, device=dev)
        N.check(L.fsc_csr_transpose(N.ptr(row_ptr), N.ptr(src), num_atoms, E, N.ptr(tr_ptr), N.ptr(tr_eid),
                                    N.ptr(ws), ws_bytes, N.stream_ptr(dev)), "fsc_csr_transpose")
        return tr_ptr, tr_eid[:E]

    @classmethod
    def from_edges(cls, edge_src, edge_dst, edge_shifts, num_atoms: int):
        dev = edge_src.device
        order = torch.argsort(edge_dst, stable=True)
        dst_sorted = edge_dst[order]
        counts = torch.bincount(dst_sorted, minlength=num_atoms)
        row_ptr = torch.zeros(num_atoms + 1, dtype=torch.int32, device=dev)
        row_ptr[1:] = torch.cumsum(counts, 0).to(torch.int32)
        src = edge_src[order].to(torch.int32).contiguous()
        shift = edge_shifts[order].to(torch.float32).contiguous()
        tr_ptr, tr_eid = cls.transpose(row_ptr, src, num_atoms)
        return cls(num_atoms, row_ptr, src, shift, tr_ptr, tr_eid, order)


class ICTDEngine:
    """Native energy + forces for one packed model (reused across calls)."""

    def __init__(self, state_dict: Dict[str, torch.Tensor], cfg: ICTDConfig, device="cuda"):
        self.cfg = cfg
        self.device = torch.device(device)
        self.ncfg = cfg.native()
        self.weights = PackedICTDWeights(state_dict, cfg, self.device)
        self._ws = None

    def workspace(self, num_atoms: int, num_edges: int):
        need = N.lib().fsc_ictd_workspace_bytes(C.byref(self.ncfg), num_atoms, num_edges)
        if need == 0:
            N.check(1, "fsc_ictd_workspace_bytes (unsupported configuration)")
        if self._ws is None or self._ws.numel() < need:
            self._ws = None
            self._ws = torch.empty(need, dtype=torch.uint8, device=self.device)
        return self._ws

    def _graph(self, pos, species, batch, cell, g: GraphCSR, num_graphs, num_local, energy_weight, field=None,
               layer_atoms=None):
        s = N.Graph()
        s.num_atoms = g.num_atoms
        s.num_local = g.num_atoms if num_local is None else int(num_local)
        s.num_edges = g.num_edges
        s.num_graphs = int(num_graphs)
        s.pos, s.species, s.batch, s.cell = pos.data_ptr(), species.data_ptr(), batch.data_ptr(), cell.data_ptr()
        s.row_ptr, s.src, s.shift = g.row_ptr.data_ptr(), g.src.data_ptr(), g.shift.data_ptr()
        s.tr_ptr, s.tr_eid = g.tr_ptr.data_ptr(), g.tr_eid.data_ptr()
        s.energy_weight = 0 if energy_weight is None else energy_weight.data_ptr()
        s.field = 0 if field is None else field.data_ptr()
        if layer_atoms is None:
            s.layer_atoms = 0
        else:
            vals = [int(v) for v in layer_atoms]
            if len(vals) != self.cfg.num_interaction:
                raise ValueError(f"layer_atoms needs {self.cfg.num_interaction} entries, got {len(vals)}")
            self._layer_arr = (C.c_int64 * len(vals))(*vals)  # host array, alive until the next call
            s.layer_atoms = C.cast(self._layer_arr, N.P)
        return s

    def _field(self, field, B):
        """(B, 3) Cartesian external field -> the conv1 l = 1 term (o3 model), or None."""
        if field is None:
            return None
        if not self.cfg.o3:
            raise ValueError("an external field needs the o3 model (ICTDConfig(o3=True))")
        f = torch.as_tensor(field, device=self.device, dtype=torch.float64).reshape(-1, 3)
        if f.shape[0] == 1 and B > 1:
            f = f.expand(B, 3)
        if f.shape[0] != B:
            raise ValueError(f"field must have one vector per graph ({B}), got {tuple(f.shape)}")
        M = T.field_l1_map().to(device=self.device)
        return (self.weights.field_scale * (f @ M.T)).to(torch.float32).contiguous()

    @staticmethod
    def _inputs(pos, species, batch, cell):
        pos = pos.detach().to(torch.float32).contiguous()
        species = species.to(torch.int32).contiguous()
        batch = batch.to(torch.int32).contiguous()
        cell = cell.detach().to(torch.float32).reshape(-1, 3, 3).contiguous()
        return pos, species, batch, cell

    def forward(self, pos, species, batch, cell, g: GraphCSR, num_local=None, field=None, layer_atoms=None):
        """Per-graph energy (B,) and per-atom energy (N,); intermediates stay in the workspace.
        ``field`` (B, 3): external 1o field of the o3 model (one Cartesian vector per graph).
        ``layer_atoms`` (num_interaction ints): receptive-field restriction of a decomposition rank
        (layer k evaluated for receiving atoms ``[0, layer_atoms[k])``; see :func:`layer_shells`)."""
        pos, species, batch, cell = self._inputs(pos, species, batch, cell)
        B = cell.shape[0]
        ws = self.workspace(g.num_atoms, g.num_edges)
        energy = torch.empty(B, dtype=torch.float32, device=self.device)
        atom_e = torch.empty(g.num_atoms, dtype=torch.float32, device=self.device)
        fdev = self._field(field, B)
        gs = self._graph(pos, species, batch, cell, g, B, num_local, None, fdev, layer_atoms)
        N.check(N.lib().fsc_ictd_forward(C.byref(self.ncfg), C.byref(self.weights.struct), C.byref(gs),
                                         N.ptr(energy), N.ptr(atom_e), N.ptr(ws), ws.numel(),
                                         N.stream_ptr(self.device)), "fsc_ictd_forward")
        self._last = (pos, species, batch, cell, g, num_local)
        self._last_layers = layer_atoms
        self._field_dev = fdev
        return energy, atom_e

    def feature_buffer(self, which: int, layer: int):
        """View (num_atoms, 9, C) of layer ``layer``'s node features (which = 0) or of their
        gradient (which = 1) in the workspace of the last call (rows l^2 + m, channel innermost)."""
        g = self._last[4]
        ws = self.workspace(g.num_atoms, g.num_edges)
        addr = C.c_void_p(0)
        N.check(N.lib().fsc_ictd_feature_buffer(C.byref(self.ncfg), g.num_atoms, g.num_edges, N.ptr(ws), which,
                                                layer, C.byref(addr)), "fsc_ictd_feature_buffer")
        off = int(addr.value) - ws.data_ptr()
        nbytes = g.num_atoms * 9 * self.cfg.channels * 4
        return ws[off:off + nbytes].view(torch.float32).view(g.num_atoms, 9, self.cfg.channels)

    def begin_steps(self, pos, species, batch, cell, g: GraphCSR, num_local=None, field=None, layer_atoms=None):
        """Set up a stepwise evaluation (:meth:`forward_step` / :meth:`backward_step`)."""
        pos, species, batch, cell = self._inputs(pos, species, batch, cell)
        B = cell.shape[0]
        self.workspace(g.num_atoms, g.num_edges)
        fdev = self._field(field, B)
        self._last = (pos, species, batch, cell, g, num_local)
        self._last_layers = layer_atoms
        self._field_dev = fdev
        self._step_out = (torch.empty(B, dtype=torch.float32, device=self.device),
                          torch.empty(g.num_atoms, dtype=torch.float32, device=self.device))

    def forward_step(self, step: int):
        """Forward step ``step`` (0 = edges + conv1, k = conv2 layer k, num_interaction = readout);
        returns (energy, atom_energy) after the last step, else layer ``step``'s feature view."""
        pos, species, batch, cell, g, num_local = self._last
        ws = self.workspace(g.num_atoms, g.num_edges)
        energy, atom_e = self._step_out
        gs = self._graph(pos, species, batch, cell, g, cell.shape[0], num_local, None, self._field_dev,
                         self._last_layers)
        last = step == self.cfg.num_interaction
        N.check(N.lib().fsc_ictd_forward_step(C.byref(self.ncfg), C.byref(self.weights.struct), C.byref(gs), step,
                                              N.ptr(energy) if last else None, N.ptr(atom_e) if last else None,
                                              N.ptr(ws), ws.numel(), N.stream_ptr(self.device)),
                f"fsc_ictd_forward_step({step})")
        return (energy, atom_e) if last else self.feature_buffer(0, step)

    def begin_backward(self, energy_weight=None, want_virial=True, want_cell_grad=False, want_edge_grad=False):
        g, B = self._last[4], self._last[3].shape[0]
        out, o = self._outputs(g, B, want_virial, want_cell_grad, want_edge_grad)
        if energy_weight is not None:
            energy_weight = energy_weight.detach().to(torch.float32).reshape(-1).contiguous()
        self._bwd = (out, o, energy_weight)
        return out

    def backward_step(self, step: int):
        """Backward step ``step`` (num_interaction = readout, k = conv2 layer k, 0 = conv1 + edges);
        returns the gradient view of layer ``step - 1`` (complete once this step ran) for
        ``step >= 1``, else the outputs."""
        pos, species, batch, cell, g, num_local = self._last
        ws = self.workspace(g.num_atoms, g.num_edges)
        out, o, ew = self._bwd
        gs = self._graph(pos, species, batch, cell, g, cell.shape[0], num_local, ew, self._field_dev,
                         self._last_layers)
        N.check(N.lib().fsc_ictd_backward_step(C.byref(self.ncfg), C.byref(self.weights.struct), C.byref(gs), step,
                                               C.byref(o), N.ptr(ws), ws.numel(), N.stream_ptr(self.device)),
                f"fsc_ictd_backward_step({step})")
        return self.feature_buffer(1, step - 1) if step >= 1 else out

    def forward_layers(self, pos, species, batch, cell, g: GraphCSR, on_layer, num_local=None, field=None,
                       layer_atoms=None):
        """:meth:`forward` in steps: after interaction layer k's features are written,
        ``on_layer(k, feats)`` may rewrite ``feats`` (a (num_atoms, 9, C) view, see
        :meth:`feature_buffer`) in place on the current stream before layer k + 1 reads them (the
        reference's sync_after_scatter points, ``pure_cartesian_ictd_layers_full.py:923-953``)."""
        self.begin_steps(pos, species, batch, cell, g, num_local, field, layer_atoms)
        nint = self.cfg.num_interaction
        for step in range(nint):
            on_layer(step, self.forward_step(step))
        return self.forward_step(nint)

    def backward_layers(self, on_grad, energy_weight=None, want_virial=True, want_cell_grad=False,
                        want_edge_grad=False):
        """:meth:`backward` in steps: before the reverse pass of interaction layer k reads the
        complete gradient of layer k's features, ``on_grad(k, grads)`` may rewrite it in place
        (the adjoint of the forward's ``on_layer``)."""
        self.begin_backward(energy_weight, want_virial, want_cell_grad, want_edge_grad)
        nint = self.cfg.num_interaction
        for step in range(nint, -1, -1):
            if step < nint:
                on_grad(step, self.feature_buffer(1, step))
            out = self.backward_step(step)
        return out

    def _outputs(self, g, B, want_virial, want_cell_grad, want_edge_grad):
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
        return out, o

    def heads(self):
        """Physical-tensor heads of the last forward (o3 model): {name: {l: (B, 1, 2l+1)}}."""
        w = self.weights
        if not w.heads:
            return {}
        pos, species, batch, cell, g, num_local = self._last
        B = cell.shape[0]
        ws = self.workspace(g.num_atoms, g.num_edges)
        nh = len(w.heads)
        out = torch.empty(nh, B, 5, dtype=torch.float32, device=self.device)
        blocks = (C.c_int32 * nh)(*[blk for _, _, blk in w.heads])
        gs = self._graph(pos, species, batch, cell, g, B, num_local, None, self._field_dev, self._last_layers)
        N.check(N.lib().fsc_ictd_heads(C.byref(self.ncfg), C.byref(w.struct), C.byref(gs), nh,
                                       C.cast(blocks, N.P), N.ptr(w.tensors["heads_w"]), N.ptr(out), N.ptr(ws),
                                       ws.numel(), N.stream_ptr(self.device)), "fsc_ictd_heads")
        res = {}
        for h, (name, l, _) in enumerate(w.heads):
            res.setdefault(name, {})[l] = out[h, :, : 2 * l + 1].reshape(B, 1, 2 * l + 1)
        return res

    def backward(self, energy_weight=None, want_virial=True, want_cell_grad=False, want_edge_grad=False):
        """Reverse pass of the last forward: forces (N,3), virial (B,3,3), dE/dcell, dE/dr."""
        pos, species, batch, cell, g, num_local = self._last
        B = cell.shape[0]
        ws = self.workspace(g.num_atoms, g.num_edges)
        dev = self.device
        out, o = self._outputs(g, B, want_virial, want_cell_grad, want_edge_grad)
        if energy_weight is not None:
            energy_weight = energy_weight.detach().to(torch.float32).reshape(-1).contiguous()
        gs = self._graph(pos, species, batch, cell, g, B, num_local, energy_weight, getattr(self, "_field_dev", None),
                         getattr(self, "_last_layers", None))
        N.check(N.lib().fsc_ictd_backward(C.byref(self.ncfg), C.byref(self.weights.struct), C.byref(gs), C.byref(o),
                                          N.ptr(ws), ws.numel(), N.stream_ptr(dev)), "fsc_ictd_backward")
        return out

    def status(self) -> int:
        """Device status word of the last call (0 = ok); synchronises the stream."""
        pos, species, batch, cell, g, num_local = self._last
        ws = self.workspace(g.num_atoms, g.num_edges)
        st = C.c_int(0)
        N.check(N.lib().fsc_ictd_status(C.byref(self.ncfg), g.num_atoms, g.num_edges, N.ptr(ws),
                                        N.stream_ptr(self.device), C.byref(st)), "fsc_ictd_status")
        return int(st.value)

    def energy_forces(self, pos, species, batch, cell, g: GraphCSR, num_local=None, want_stress=True, field=None):
        energy, atom_e = self.forward(pos, species, batch, cell, g, num_local, field)
        out = self.backward(want_virial=want_stress)
        out["energy"] = energy
        out["atom_energy"] = atom_e
        if want_stress:
            vol = torch.abs(torch.det(self._last[3].double())).clamp(min=1e-10).float()
            v = out["virial"]
            out["stress"] = 0.5 * (v + v.transpose(1, 2)) / vol.view(-1, 1, 1)
        return out
