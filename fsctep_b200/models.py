"""Drop-in ``PureCartesianICTDTransformerLayer`` (``--tensor-product-mode pure-cartesian-ictd``).

Same constructor arguments, submodule names and ``state_dict`` keys/shapes as the reference
``models/pure_cartesian_ictd_layers_full.py:476-866``, so a reference checkpoint loads with
``load_state_dict``.  ``forward`` has the reference signature (``:867-886``) and returns the
per-atom energy ``(N, 1)``; it is differentiable w.r.t. ``pos`` and ``cell`` through a custom
autograd function whose backward is the native hand-written reverse pass (forces, and the
cell gradient that the trainer's strain-based stress needs), so
``torch.autograd.grad(E, pos)`` works as in ``evaluation/calculator.py:158-159``.

Covered: lmax 2, path policy "full", channels 32/64, gaussian or bessel radial basis,
no external tensor, no physical-tensor heads, no long-range / spectral modules.  With
``precomputed_edge_vec`` (the LAMMPS ML-IAP call, ``interfaces/lammps_mliap.py:395-420, 745-760``)
the energy depends on the given edge vectors only and is differentiable in them.
``sync_after_scatter`` (``cli/inference_ddp.py:143-340``) is called after conv1 and after every
conv2 scatter on the node features in the reference layout, through the engine's stepwise
evaluation, and its vector-Jacobian product enters the native reverse pass.  Anything else raises
``NotImplementedError`` (there is no CPU path to fall back to).
"""

from __future__ import annotations

from typing import Dict, Optional

import torch
import torch.nn as nn

from fsctep_b200.ictd import ICTDConfig, ICTDEngine, GraphCSR
from fsctep_b200.tables import paths_full


class _TP(nn.Module):
    def __init__(self, num_paths, mul_out, mul_in1, mul_in2):
        super().__init__()
        self.weight = nn.Parameter(torch.randn(num_paths, mul_out, mul_in1, mul_in2) * 0.02)
        self.num_paths = num_paths


def _radial_mlp(nb, num_paths):
    return nn.Sequential(nn.Linear(nb, 64), nn.SiLU(), nn.Linear(64, 64), nn.SiLU(), nn.Linear(64, num_paths))


class _Conv1(nn.Module):
    def __init__(self, cfg: ICTDConfig, num_paths):
        super().__init__()
        self.atom_embedding = nn.Embedding(cfg.max_atomvalue, cfg.embedding_dim)
        self.atom_mlp = nn.Sequential(nn.Linear(cfg.embedding_dim, 64), nn.SiLU(), nn.Linear(64, cfg.output_size))
        self.tp2 = _TP(num_paths, cfg.channels, cfg.output_size, cfg.output_size)
        self.fc = _radial_mlp(cfg.number_of_basis, num_paths)


class _MainNet(nn.Module):
    def __init__(self, input_size, hidden_sizes, output_size):
        super().__init__()
        self.layers = nn.ModuleList()
        self.layer_norms = nn.ModuleList()
        self.input_norm = nn.LayerNorm(input_size)
        sizes = [input_size] + list(hidden_sizes)
        for a, b in zip(sizes[:-1], sizes[1:]):
            self.layers.append(nn.Linear(a, b))
            self.layer_norms.append(nn.LayerNorm(b))
        self.output = nn.Linear(sizes[-1], output_size)
        self.input_size = input_size


class _WeightedSum(nn.Module):
    def __init__(self, n):
        super().__init__()
        self.weights = nn.Parameter(torch.zeros(n))


class _NativeEnergy(torch.autograd.Function):
    """Per-atom energy of the native engine, differentiable in ``pos`` and ``cell`` -- or, with
    ``edge_vec`` (the reference's ``precomputed_edge_vec``, ``pure_cartesian_ictd_layers_full.py:
    901-902``), in the given edge vectors only: the engine then sees zero positions, identity cells
    and shift = edge_vec, so r_e = edge_vec exactly, and dE/d(edge_vec) is its per-edge dE/dr_e in
    the caller's edge order.  ``hook`` is the reference's ``sync_after_scatter``: it is called on
    every layer's node features in the reference layout and its vector-Jacobian product is
    applied to their gradient in the reverse pass."""

    @staticmethod
    def forward(ctx, pos, cell, edge_vec, owner, graph, species, batch, field, hook):
        eng = owner._engine
        ctx.owner, ctx.graph, ctx.species, ctx.batch, ctx.field, ctx.hook = owner, graph, species, batch, field, hook
        ctx.num_graphs = cell.shape[0]
        ctx.edge_mode = edge_vec is not None
        ctx.hook_io = []
        _, atom_e = _run_forward(ctx, pos, cell, replay=False)
        ctx.generation = owner._bump()
        ctx.save_for_backward(pos, cell)
        ctx.out_dtype = (edge_vec if ctx.edge_mode else pos).dtype
        ctx.pos_dtype, ctx.cell_dtype = pos.dtype, cell.dtype
        return atom_e.view(-1, 1).to(ctx.out_dtype)

    @staticmethod
    def backward(ctx, grad_e):
        pos, cell = ctx.saved_tensors
        owner, g = ctx.owner, ctx.graph
        eng = owner._engine
        if owner._generation != ctx.generation:  # another forward reused the workspace: recompute
            _run_forward(ctx, pos, cell, replay=True)
            owner._generation = ctx.generation
        want_cell = (not ctx.edge_mode) and ctx.needs_input_grad[1]
        kw = dict(energy_weight=grad_e.reshape(-1), want_virial=False, want_cell_grad=want_cell,
                  want_edge_grad=ctx.edge_mode)
        if ctx.hook is None:
            out = eng.backward(**kw)
        else:
            blocks = owner._ref_blocks()

            def on_grad(k, grads):
                x, y = ctx.hook_io[k]
                if not y.requires_grad:  # the hook cut the graph: nothing flows back through it
                    grads.zero_()
                    return
                (gx,) = torch.autograd.grad(y, x, _native_to_ref(grads, blocks).to(y.dtype))
                _ref_to_native(gx, blocks, grads)

            out = eng.backward_layers(on_grad, **kw)
        gpos = gcell = gvec = None
        if ctx.edge_mode:
            gvec = torch.empty_like(out["edge_grad"])
            gvec[g.order] = out["edge_grad"]
            gvec = gvec.to(ctx.out_dtype)
        else:
            gpos = (-out["forces"]).to(ctx.pos_dtype) if ctx.needs_input_grad[0] else None
            gcell = out["cell_grad"].to(ctx.cell_dtype).reshape(cell.shape) if want_cell else None
        return gpos, gcell, gvec, None, None, None, None, None, None


def _run_forward(ctx, pos, cell, replay):
    """The engine's forward for the autograd function; with a hook, the hook's inputs and outputs
    are kept for the reverse pass (a replay after the workspace was reused writes the kept outputs
    again instead of calling the hook, which may hold collectives, a second time)."""
    eng = ctx.owner._engine
    if ctx.edge_mode:
        pos, cell = _edge_vec_frame(ctx.species.shape[0], ctx.num_graphs, ctx.species.device)
    if ctx.hook is None:
        return eng.forward(pos, ctx.species, ctx.batch, cell, ctx.graph, field=ctx.field)
    blocks = ctx.owner._ref_blocks()

    def on_layer(k, feats):
        if replay:
            _ref_to_native(ctx.hook_io[k][1].detach(), blocks, feats)
            return
        x = _native_to_ref(feats, blocks).requires_grad_(True)
        with torch.enable_grad():
            y = ctx.hook(x)
        if not isinstance(y, torch.Tensor) or y.shape != x.shape:
            raise ValueError(f"sync_after_scatter must return a tensor of shape {tuple(x.shape)}")
        ctx.hook_io.append((x, y))
        _ref_to_native(y.detach(), blocks, feats)

    return eng.forward_layers(pos, ctx.species, ctx.batch, cell, ctx.graph, on_layer, field=ctx.field)


def _native_to_ref(feats, blocks):
    """(N, 9, C) native rows (l^2 + m, channel innermost) -> the reference's flat per-node layout:
    per irrep block, channel-major (C, 2l + 1) (``_merge_irreps``); blocks without native storage
    (the o3 model's 1e, identically zero) are zeros."""
    n, _, c = feats.shape
    parts = []
    for r0, m in blocks:
        if r0 is None:
            parts.append(feats.new_zeros(n, c * m))
        else:
            parts.append(feats[:, r0:r0 + m, :].transpose(1, 2).reshape(n, c * m))
    return torch.cat(parts, dim=-1)


def _ref_to_native(x, blocks, feats):
    """Inverse of :func:`_native_to_ref`, written into ``feats`` in place (zero blocks skipped)."""
    n, _, c = feats.shape
    off = 0
    for r0, m in blocks:
        if r0 is not None:
            feats[:, r0:r0 + m, :] = x[:, off:off + c * m].reshape(n, c, m).transpose(1, 2).to(feats.dtype)
        off += c * m


def _edge_vec_frame(n, num_graphs, device):
    """Zero positions and identity cells: with shift = edge_vec the engine's r_e is edge_vec."""
    pos0 = torch.zeros(n, 3, dtype=torch.float32, device=device)
    eye = torch.eye(3, dtype=torch.float32, device=device).expand(num_graphs, 3, 3).contiguous()
    return pos0, eye


def _edge_vec_graph(edge_src, edge_dst, edge_vec, n):
    if edge_vec.shape != (edge_src.shape[0], 3):
        raise ValueError(f"precomputed_edge_vec must be (E, 3) = ({edge_src.shape[0]}, 3), got {tuple(edge_vec.shape)}")
    if not edge_vec.is_cuda:
        raise RuntimeError("fsctep_b200 runs on CUDA devices only (no CPU path)")
    return GraphCSR.from_edges(edge_src.long(), edge_dst.long(), edge_vec.detach(), n)


class PureCartesianICTDTransformerLayer(nn.Module):
    def __init__(self, max_embed_radius: float, main_max_radius: float, main_number_of_basis: int,
                 hidden_dim_conv: int, hidden_dim_sh=None, hidden_dim=None, channel_in2: int = 32,
                 embedding_dim: int = 16, max_atomvalue: int = 10, output_size: int = 8, embed_size=None,
                 main_hidden_sizes3=None, num_layers: int = 1, num_interaction: int = 2, device=None,
                 function_type_main: str = "gaussian", lmax: int = 2, ictd_Lmax: int = 6,
                 ictd_tp_path_policy: str = "full", ictd_tp_max_rank_other=None, max_rank_other: int = 1,
                 k_policy: str = "k0", internal_compute_dtype=None, ictd_tp_backend: str = "auto",
                 product5_muls_by_l=None, invariant_channels: int = 32, physical_tensor_outputs=None,
                 external_tensor_rank=None, external_tensor_irrep=None, external_tensor_parity=None,
                 external_tensor_specs=None, num_fidelity_levels: int = 0, long_range_mode: str = "none",
                 feature_spectral_mode: str = "none", **unused):
        super().__init__()
        if embed_size is None:
            embed_size = [128, 128, 128]
        unsupported = []
        if ictd_tp_path_policy != "full":
            unsupported.append(f"ictd_tp_path_policy={ictd_tp_path_policy!r}")
        if int(lmax) != 2:
            unsupported.append(f"lmax={lmax}")
        if product5_muls_by_l is not None:
            unsupported.append("product5_muls_by_l")
        if physical_tensor_outputs:
            unsupported.append("physical_tensor_outputs")
        if external_tensor_rank is not None or external_tensor_specs:
            unsupported.append("external tensors")
        if num_fidelity_levels:
            unsupported.append("multi-fidelity")
        if long_range_mode != "none" or feature_spectral_mode != "none":
            unsupported.append("long-range / spectral modules")
        if int(num_interaction) < 2:
            raise ValueError(f"num_interaction must be >= 2, got {num_interaction}")
        if unsupported:
            raise NotImplementedError("fsctep_b200 pure-cartesian-ictd does not cover: " + ", ".join(unsupported))
        self.cfg = ICTDConfig(channels=int(hidden_dim_conv), lmax=int(lmax), num_interaction=int(num_interaction),
                              number_of_basis=int(main_number_of_basis), max_radius=float(max_embed_radius),
                              function_type=str(function_type_main), output_size=int(output_size),
                              embedding_dim=int(embedding_dim), max_atomvalue=int(max_atomvalue),
                              invariant_channels=int(invariant_channels), embed_size=tuple(embed_size))
        self.cfg.native()  # validates the radial basis kind
        self.lmax = int(lmax)
        self.channels = int(hidden_dim_conv)
        self.num_interaction = int(num_interaction)
        self.max_radius = float(max_embed_radius)
        self.number_of_basis = int(main_number_of_basis)
        self.function_type = str(function_type_main)
        self.invariant_channels = int(invariant_channels)
        P = len(paths_full(self.lmax))
        C, nint = self.channels, self.num_interaction
        self.e3_conv_emb = _Conv1(self.cfg, P)
        self.tp2_layers = nn.ModuleList([_TP(P, C, C, 1) for _ in range(nint - 1)])
        self.fc2_layers = nn.ModuleList([_radial_mlp(self.number_of_basis, P) for _ in range(nint - 1)])
        nC = C * nint
        S = (nint - 1) * self.invariant_channels
        self.W_read = nn.ParameterList([nn.Parameter(torch.randn(S, nC, nC) * 0.02) for _ in range(self.lmax + 1)])
        self.readout_linear = nn.Sequential(nn.Linear(S + (self.lmax + 1) * nC, embed_size[0]), nn.SiLU(),
                                            nn.Linear(embed_size[0], 17))
        self.weighted_sum = _WeightedSum(17)
        self.proj_total = _MainNet(nint * (self.lmax + 1) * C + S, embed_size, 17)
        self._engine: Optional[ICTDEngine] = None
        self._engine_key = None
        self._generation = 0

    def _bump(self):
        self._generation += 1
        return self._generation

    def _ref_blocks(self):
        """(native first row or None, 2l + 1) per irrep block of the reference feature layout."""
        return [(0, 1), (1, 3), (4, 5)]

    def _ensure_engine(self, device):
        key = (str(device),) + tuple((p.data_ptr(), p._version) for p in self.parameters())
        if self._engine is None or self._engine_key != key:
            self._engine = ICTDEngine({k: v.detach() for k, v in self.state_dict().items()}, self.cfg, device)
            self._engine_key = key
        return self._engine

    def forward(self, pos, A, batch, edge_src, edge_dst, edge_shifts, cell, *, precomputed_edge_vec=None,
                sync_after_scatter=None, external_tensor=None, external_tensor_blocks=None, fidelity_ids=None,
                return_physical_tensors: bool = False, return_reciprocal_source: bool = False):
        if external_tensor is not None or external_tensor_blocks is not None or return_physical_tensors \
                or return_reciprocal_source:
            raise NotImplementedError("fsctep_b200 pure-cartesian-ictd forward covers (pos, A, batch, edges, cell), "
                                      "precomputed_edge_vec and sync_after_scatter")
        if not pos.is_cuda:
            raise RuntimeError("fsctep_b200 runs on CUDA devices only (no CPU path)")
        n = pos.shape[0]
        species = A.long()
        if n and int(species.max().item()) >= self.cfg.max_atomvalue:
            raise IndexError("atomic number out of range of atom_embedding (max_atomvalue)")
        cell = cell.reshape(-1, 3, 3)
        if n and int(batch.max().item()) >= cell.shape[0]:
            raise IndexError("batch index out of range of cell")
        self._ensure_engine(pos.device)
        if precomputed_edge_vec is not None:
            graph = _edge_vec_graph(edge_src, edge_dst, precomputed_edge_vec, n)
        else:
            graph = GraphCSR.from_edges(edge_src.long(), edge_dst.long(), edge_shifts, n)
        return _NativeEnergy.apply(pos, cell, precomputed_edge_vec, self, graph, species, batch, None,
                                   sync_after_scatter)


_O3_IRREPS = {("0e", "1o", "2e"), ("0e", "1e", "1o", "2e")}


def _irrep_letter(l: int, p: int) -> str:
    return f"{l}{'e' if p > 0 else 'o'}"


class PureCartesianICTDO3TransformerLayer(nn.Module):
    """Drop-in for ``PureCartesianICTDO3TransformerLayer`` (``--tensor-product-mode
    pure-cartesian-ictd-o3``, ``models/pure_cartesian_ictd_layers_o3.py:535-1074``).

    Same constructor, parameter names and shapes, and forward signature.  Covered: lmax 2, active
    irreps 0e,1o,2e (preset "auto") or 0e,1e,1o,2e, an optional rank-1 external field (1o, one
    vector per graph or one for all), dipole / polarizability-style heads (bias-free linear maps of
    the readout blocks, reduce "sum").  The energy is differentiable in ``pos`` and ``cell``
    through the native reverse pass; the physical-tensor outputs are returned without a graph."""

    def __init__(self, max_embed_radius: float, main_max_radius: float, main_number_of_basis: int,
                 hidden_dim_conv: int, hidden_dim_sh=None, hidden_dim=None, channel_in2: int = 32,
                 embedding_dim: int = 16, max_atomvalue: int = 10, output_size: int = 8, embed_size=None,
                 main_hidden_sizes3=None, num_layers: int = 1, num_interaction: int = 2, device=None,
                 function_type_main: str = "gaussian", lmax: int = 2, ictd_tp_path_policy: str = "full",
                 ictd_tp_max_rank_other=None, internal_compute_dtype=None, ictd_tp_backend: str = "auto",
                 invariant_channels: int = 32, physical_tensor_outputs=None, external_tensor_rank=None,
                 external_tensor_irrep=None, external_tensor_parity=None, external_tensor_specs=None,
                 o3_irrep_preset: str = "auto", o3_active_irreps=None, num_fidelity_levels: int = 0,
                 long_range_mode: str = "none", feature_spectral_mode: str = "none",
                 external_tensor_scale_init: float = 0.0, **unused):
        super().__init__()
        if embed_size is None:
            embed_size = [128, 128, 128]
        unsupported = []
        if ictd_tp_path_policy != "full" or int(lmax) != 2:
            unsupported.append("lmax != 2 or a path policy other than 'full'")
        if external_tensor_specs or (external_tensor_rank is not None and int(external_tensor_rank) != 1):
            unsupported.append("external tensors other than one rank-1 field")
        if external_tensor_rank is not None and external_tensor_irrep not in (None, "1o") and \
                external_tensor_parity not in (None, "o", -1):
            unsupported.append("a 1e external field")
        if num_fidelity_levels or long_range_mode != "none" or feature_spectral_mode != "none":
            unsupported.append("multi-fidelity / long-range / spectral modules")
        if o3_active_irreps is not None:
            irreps = tuple(sorted({str(x).strip() for x in o3_active_irreps} | {"0e"},
                                  key=lambda t: (int(t[0]), t[1] == "o")))
        elif str(o3_irrep_preset).lower() in ("auto", "minimal"):
            irreps = ("0e", "1o", "2e")
        else:
            irreps = ()
        if irreps not in _O3_IRREPS:
            unsupported.append(f"active irreps {irreps or o3_irrep_preset!r}")
        heads = {}
        for name, spec in (physical_tensor_outputs or {}).items():
            if str(spec.get("reduce", "sum")).lower() != "sum" or spec.get("channels_out", 1) != 1:
                unsupported.append(f"physical tensor head {name!r} (reduce 'sum', channels_out 1 only)")
                continue
            if spec.get("irreps") is not None:
                ir = [str(x) for x in spec["irreps"]]
            else:
                ir = [_irrep_letter(int(l), 1 if int(l) % 2 == 0 else -1) for l in spec.get("ls", [])]
            if any(x not in irreps for x in ir):
                unsupported.append(f"physical tensor head {name!r} on inactive irreps")
            heads[name] = ir
        if unsupported:
            raise NotImplementedError("fsctep_b200 pure-cartesian-ictd-o3 does not cover: " + ", ".join(unsupported))
        if int(num_interaction) < 2:
            raise ValueError(f"num_interaction must be >= 2, got {num_interaction}")
        self.irreps = irreps
        self.cfg = ICTDConfig(channels=int(hidden_dim_conv), lmax=2, num_interaction=int(num_interaction),
                              number_of_basis=int(main_number_of_basis), max_radius=float(max_embed_radius),
                              function_type=str(function_type_main), output_size=int(output_size),
                              embedding_dim=int(embedding_dim), max_atomvalue=int(max_atomvalue),
                              invariant_channels=int(invariant_channels), embed_size=tuple(embed_size),
                              o3=True, o3_irreps=irreps)
        self.cfg.native()
        C, nint = int(hidden_dim_conv), int(num_interaction)
        from fsctep_b200.ictd import o3_num_paths

        P = o3_num_paths(irreps)
        self.channels, self.num_interaction = C, nint
        self.e3_conv_emb = _Conv1(self.cfg, P)
        if external_tensor_rank is not None:
            self.e3_conv_emb.external_tensor_scale_by_irrep = nn.Parameter(
                torch.full((len(irreps),), float(external_tensor_scale_init)))
        self.external_tensor_rank = external_tensor_rank
        self.tp2_layers = nn.ModuleList([_TP(P, C, C, 1) for _ in range(nint - 1)])
        self.fc2_layers = nn.ModuleList([_radial_mlp(int(main_number_of_basis), P) for _ in range(nint - 1)])
        nC = C * nint
        S = (nint - 1) * int(invariant_channels)
        self.W_read = nn.ParameterDict({k: nn.Parameter(torch.randn(S, nC, nC) * 0.02) for k in irreps})
        self.readout_linear = nn.Sequential(nn.Linear(S + nC * len(irreps), embed_size[0]), nn.SiLU(),
                                            nn.Linear(embed_size[0], 17))
        self.weighted_sum = _WeightedSum(17)
        self.proj_total = _MainNet(nint * C * len(irreps) + S, embed_size, 17)
        self._head_spec = heads
        if heads:
            self.physical_tensor_heads = nn.ModuleDict({
                name: nn.ModuleDict({ir[0]: nn.Linear(nC, 1, bias=False) for ir in irs})
                for name, irs in heads.items()})
        else:
            self.physical_tensor_heads = None
        self._engine: Optional[ICTDEngine] = None
        self._engine_key = None
        self._generation = 0

    _bump = PureCartesianICTDTransformerLayer._bump
    _ensure_engine = PureCartesianICTDTransformerLayer._ensure_engine

    def _ref_blocks(self):
        # reference irrep order (l, even before odd): 0e, [1e,] 1o, 2e; the native rows hold
        # 0e, 1o, 2e (1e couples only to itself and stays zero without a 1e input)
        rows = {"0e": (0, 1), "1e": (None, 3), "1o": (1, 3), "2e": (4, 5)}
        return [rows[k] for k in self.irreps]

    def forward(self, pos, A, batch, edge_src, edge_dst, edge_shifts, cell, *, precomputed_edge_vec=None,
                sync_after_scatter=None, external_tensor=None, fidelity_ids=None,
                return_physical_tensors: bool = False, return_reciprocal_source: bool = False):
        if return_reciprocal_source or fidelity_ids is not None:
            raise NotImplementedError("fsctep_b200 pure-cartesian-ictd-o3 forward: optional inputs other than "
                                      "precomputed_edge_vec / sync_after_scatter / external_tensor / "
                                      "return_physical_tensors are not covered")
        if not pos.is_cuda:
            raise RuntimeError("fsctep_b200 runs on CUDA devices only (no CPU path)")
        n = pos.shape[0]
        species = A.long()
        if n and int(species.max().item()) >= self.cfg.max_atomvalue:
            raise IndexError("atomic number out of range of atom_embedding (max_atomvalue)")
        cell = cell.reshape(-1, 3, 3)
        field = None
        if external_tensor is not None:
            if self.external_tensor_rank is None:
                raise ValueError("external_tensor given but the model has no external tensor input")
            field = external_tensor.detach().reshape(-1, 3)
        eng = self._ensure_engine(pos.device)
        if precomputed_edge_vec is not None:
            graph = _edge_vec_graph(edge_src, edge_dst, precomputed_edge_vec, n)
        else:
            graph = GraphCSR.from_edges(edge_src.long(), edge_dst.long(), edge_shifts, n)
        e = _NativeEnergy.apply(pos, cell, precomputed_edge_vec, self, graph, species, batch, field,
                                sync_after_scatter)
        if not return_physical_tensors:
            return e
        if self.physical_tensor_heads is None:
            raise ValueError("return_physical_tensors=True but physical_tensor_outputs was not set in __init__")
        return e, eng.heads()


class _SparseConv1(nn.Module):
    def __init__(self, cfg, P):
        super().__init__()
        self.atom_embedding = nn.Embedding(cfg.max_atomvalue, cfg.embedding_dim)
        self.atom_mlp = nn.Sequential(nn.Linear(cfg.embedding_dim, 64), nn.SiLU(), nn.Linear(64, cfg.output_size))
        self.fc = _radial_mlp(cfg.number_of_basis, P * cfg.channels * cfg.output_size * cfg.output_size)


class _SparseConv2(nn.Module):
    def __init__(self, cfg, P):
        super().__init__()
        self.fc = _radial_mlp(cfg.number_of_basis, P * cfg.channels * cfg.channels)


class _Bilinear(nn.Module):
    def __init__(self, channels, out_channels, lmax):
        super().__init__()
        self.W = nn.ParameterList([nn.Parameter(torch.randn(out_channels, channels, channels) * 0.02)
                                   for _ in range(lmax + 1)])


class _SparseEnergy(torch.autograd.Function):
    @staticmethod
    def forward(ctx, pos, cell, owner, graph, species, batch):
        eng = owner._engine
        _, atom_e = eng.forward(pos, species, batch, cell, graph)
        ctx.owner, ctx.graph, ctx.species, ctx.batch = owner, graph, species, batch
        ctx.generation = owner._bump()
        ctx.save_for_backward(pos, cell)
        ctx.pos_dtype, ctx.cell_dtype = pos.dtype, cell.dtype
        return atom_e.view(-1, 1).to(pos.dtype)

    @staticmethod
    def backward(ctx, grad_e):
        pos, cell = ctx.saved_tensors
        owner = ctx.owner
        eng = owner._engine
        if owner._generation != ctx.generation:
            eng.forward(pos, ctx.species, ctx.batch, cell, ctx.graph)
            owner._generation = ctx.generation
        out = eng.backward(energy_weight=grad_e.reshape(-1), want_virial=False,
                           want_cell_grad=ctx.needs_input_grad[1])
        gpos = (-out["forces"]).to(ctx.pos_dtype) if ctx.needs_input_grad[0] else None
        gcell = out["cell_grad"].to(ctx.cell_dtype).reshape(cell.shape) if ctx.needs_input_grad[1] else None
        return gpos, gcell, None, None, None, None


class PureCartesianSparseTransformerLayer(nn.Module):
    """Drop-in for ``PureCartesianSparseTransformerLayer`` (``--tensor-product-mode
    pure-cartesian-sparse``, ``models/pure_cartesian_sparse_layers.py:459-855``).

    Same constructor, parameter names (``e3_conv_emb`` is ``e3_conv_layers[0]``, as in the
    reference) and forward signature; per-atom energy (N, 1) differentiable in ``pos`` and
    ``cell`` through the native reverse pass.  Covered: lmax 2 or 3, channels 32/64/128,
    max_rank_other 1, k_policy "k0", no external tensors / heads / long-range / fidelity."""

    def __init__(self, max_embed_radius: float, main_max_radius: float, main_number_of_basis: int,
                 hidden_dim_conv: int, hidden_dim_sh=None, hidden_dim=None, channel_in2: int = 32,
                 embedding_dim: int = 16, max_atomvalue: int = 10, output_size: int = 8, invariant_channels: int = 32,
                 embed_size=None, main_hidden_sizes3=None, num_layers: int = 1, num_interaction: int = 2, device=None,
                 function_type_main: str = "gaussian", lmax: int = 2, max_rank_other: int = 1, k_policy: str = "k0",
                 long_range_mode: str = "none", feature_spectral_mode: str = "none", physical_tensor_outputs=None,
                 external_tensor_rank=None, external_tensor_specs=None, num_fidelity_levels: int = 0, **unused):
        super().__init__()
        from fsctep_b200.sparse import SparseConfig, sparse_paths

        if embed_size is None:
            embed_size = [128, 128, 128]
        unsupported = []
        if int(max_rank_other) != 1 or str(k_policy) != "k0":
            unsupported.append(f"max_rank_other={max_rank_other}, k_policy={k_policy!r}")
        if int(lmax) not in (2, 3):
            unsupported.append(f"lmax={lmax}")
        if int(hidden_dim_conv) not in (32, 64, 128):
            unsupported.append(f"channels={hidden_dim_conv}")
        if physical_tensor_outputs or external_tensor_rank is not None or external_tensor_specs or num_fidelity_levels:
            unsupported.append("physical-tensor heads / external tensors / multi-fidelity")
        if long_range_mode != "none" or feature_spectral_mode != "none":
            unsupported.append("long-range / spectral modules")
        if unsupported:
            raise NotImplementedError("fsctep_b200 pure-cartesian-sparse does not cover: " + ", ".join(unsupported))
        if int(num_interaction) < 2:
            raise ValueError(f"num_interaction must be >= 2, got {num_interaction}")
        self.cfg = SparseConfig(channels=int(hidden_dim_conv), lmax=int(lmax), num_interaction=int(num_interaction),
                                number_of_basis=int(main_number_of_basis), max_radius=float(max_embed_radius),
                                function_type=str(function_type_main), output_size=int(output_size),
                                embedding_dim=int(embedding_dim), max_atomvalue=int(max_atomvalue),
                                invariant_channels=int(invariant_channels), embed_size=tuple(embed_size))
        self.cfg.native()
        C, nint, L = self.cfg.channels, self.cfg.num_interaction, self.cfg.lmax
        P = len(sparse_paths(L))
        self.channels, self.num_interaction, self.Lmax = C, nint, L
        self.e3_conv_layers = nn.ModuleList([_SparseConv1(self.cfg, P)] +
                                            [_SparseConv2(self.cfg, P) for _ in range(1, nint)])
        self.e3_conv_emb = self.e3_conv_layers[0]
        S = (nint - 1) * int(invariant_channels)
        self.product_3 = _Bilinear(C * nint, S, L)
        self.proj_total = _MainNet(nint * C * (L + 1) + S, embed_size, 17)
        self.weighted_sum = _WeightedSum(17)
        self._engine = None
        self._engine_key = None
        self._generation = 0

    _bump = PureCartesianICTDTransformerLayer._bump

    def _ensure_engine(self, device):
        from fsctep_b200.sparse import SparseEngine

        key = (str(device),) + tuple((p.data_ptr(), p._version) for p in self.parameters())
        if self._engine is None or self._engine_key != key:
            self._engine = SparseEngine({k: v.detach() for k, v in self.state_dict().items()}, self.cfg, device)
            self._engine_key = key
        return self._engine

    def forward(self, pos, A, batch, edge_src, edge_dst, edge_shifts, cell, *, precomputed_edge_vec=None,
                external_tensor=None, fidelity_ids=None, return_physical_tensors: bool = False,
                return_reciprocal_source: bool = False, **_unused):
        # The reference accepts precomputed_edge_vec here but never reads it (its forward always
        # rebuilds the edge vectors from pos, shifts and cell, pure_cartesian_sparse_layers.py:745-756),
        # and it swallows sync_after_scatter through **_unused: both are accepted and ignored alike.
        if external_tensor is not None or fidelity_ids is not None or return_physical_tensors \
                or return_reciprocal_source:
            raise NotImplementedError("fsctep_b200 pure-cartesian-sparse forward covers (pos, A, batch, edges, cell)")
        if not pos.is_cuda:
            raise RuntimeError("fsctep_b200 runs on CUDA devices only (no CPU path)")
        n = pos.shape[0]
        species = A.long()
        if n and int(species.max().item()) >= self.cfg.max_atomvalue:
            raise IndexError("atomic number out of range of atom_embedding (max_atomvalue)")
        cell = cell.reshape(-1, 3, 3)
        self._ensure_engine(pos.device)
        graph = GraphCSR.from_edges(edge_src.long(), edge_dst.long(), edge_shifts, n)
        return _SparseEnergy.apply(pos, cell, self, graph, species, batch)


def reference_state_dict_shapes(cfg: ICTDConfig) -> Dict[str, tuple]:
    """Shapes of the reference state_dict for a config (for seeded synthetic weights)."""
    with torch.device("meta"):
        m = PureCartesianICTDTransformerLayer(
            max_embed_radius=cfg.max_radius, main_max_radius=cfg.max_radius,
            main_number_of_basis=cfg.number_of_basis, hidden_dim_conv=cfg.channels, lmax=cfg.lmax,
            num_interaction=cfg.num_interaction, function_type_main=cfg.function_type,
            max_atomvalue=cfg.max_atomvalue, embedding_dim=cfg.embedding_dim, output_size=cfg.output_size,
            invariant_channels=cfg.invariant_channels, embed_size=list(cfg.embed_size))
    return {k: tuple(v.shape) for k, v in m.state_dict().items()}
