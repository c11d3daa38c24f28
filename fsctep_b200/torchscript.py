"""core.pt export: the pure-cartesian-ictd, -ictd-o3 and -sparse models as traced TorchScript
modules whose only compute is one custom op (``fsctep::ictd_atom_energy``,
``fsctep::ictd_o3_atom_energy`` with the external field, ``fsctep::sparse_atom_energy``;
torch_ops/ictd_op.cpp).

Signature and outputs follow the reference's traced core (``_TorchScriptEdgeVecCore``,
interfaces/lammps_mliap.py:372-420, exported by cli/export_libtorch_core.py):
``forward(pos, A, batch, edge_src, edge_dst, edge_shifts, cell, edge_vec, external_tensor)
-> atom_energy (N, 1)``, differentiable with respect to ``edge_vec`` (the LAMMPS engine,
mff_torch_engine.cpp:459-569, takes ``autograd::grad`` of the local energy through it).  Load the
op library before ``torch.jit.load`` (LAMMPS: ``MFF_CUSTOM_OPS_LIB=<op library path>``).

The o3 core takes the external field as the ``external_tensor`` input (3 values, the system's one
graph) and maps it to the engine's l = 1 conv1 term inside the traced graph; it returns the
per-atom energy tensor (the reference's traced core returns the physical-tensor tuple as well,
``lammps_mliap.py:218-330``; the heads stay available through the Python module).  The sparse
core evaluates the given edge vectors.  (The reference's sparse model accepts
``precomputed_edge_vec`` but never reads it, so its own traced core differentiates through the
positions and shifts; with the LAMMPS engine's ``edge_vec = pos[dst] - pos[src] + shift`` both
give the same energies and forces.)
"""

from __future__ import annotations

import json
import os
from typing import Dict, List

import torch
import torch.nn as nn

from .ictd import ICTDConfig, PackedICTDWeights, weight_blob

OPLIB = os.path.join(os.path.dirname(os.path.abspath(__file__)), "_lib", "libfsctep_b200_torch.so")
_loaded = False


def load_ops() -> str:
    """Load the op library into this process (idempotent); returns its path."""
    global _loaded
    if not _loaded:
        if not os.path.exists(OPLIB):
            raise RuntimeError(f"{OPLIB} is missing: run `python -m fsctep_b200.build`")
        torch.ops.load_library(OPLIB)
        _loaded = True
    return OPLIB


class ICTDCore(nn.Module):
    """Traceable core of one pure-cartesian-ictd model (weights packed into one buffer)."""

    def __init__(self, state_dict: Dict[str, torch.Tensor], cfg: ICTDConfig, device="cuda"):
        super().__init__()
        load_ops()
        packed = PackedICTDWeights(state_dict, cfg, device)
        blob, icfg, fcfg = weight_blob(packed, cfg)
        self.register_buffer("blob", blob)
        self.icfg: List[int] = [int(x) for x in icfg]
        self.fcfg: List[float] = [float(x) for x in fcfg]
        self.cutoff = float(cfg.max_radius)

    def forward(self, pos: torch.Tensor, A: torch.Tensor, batch: torch.Tensor, edge_src: torch.Tensor,
                edge_dst: torch.Tensor, edge_shifts: torch.Tensor, cell: torch.Tensor, edge_vec: torch.Tensor,
                external_tensor: torch.Tensor) -> torch.Tensor:
        return torch.ops.fsctep.ictd_atom_energy(edge_vec, A, edge_src, edge_dst, self.blob, self.icfg, self.fcfg)


class ICTDO3Core(ICTDCore):
    """Traceable core of one pure-cartesian-ictd-o3 model with a rank-1 external field."""

    def __init__(self, state_dict: Dict[str, torch.Tensor], cfg: ICTDConfig, device="cuda"):
        super().__init__(state_dict, cfg, device)
        from . import tables as T

        packed = PackedICTDWeights(state_dict, cfg, device)
        self.register_buffer("field_map", (packed.field_scale * T.field_l1_map()).to(torch.float32).to(device))

    def forward(self, pos: torch.Tensor, A: torch.Tensor, batch: torch.Tensor, edge_src: torch.Tensor,
                edge_dst: torch.Tensor, edge_shifts: torch.Tensor, cell: torch.Tensor, edge_vec: torch.Tensor,
                external_tensor: torch.Tensor) -> torch.Tensor:
        field = external_tensor.reshape(1, 3).to(torch.float32) @ self.field_map.T
        return torch.ops.fsctep.ictd_o3_atom_energy(edge_vec, A, edge_src, edge_dst, field, self.blob, self.icfg,
                                                    self.fcfg)


class SparseCore(nn.Module):
    """Traceable core of one pure-cartesian-sparse model (weights packed into one buffer)."""

    def __init__(self, state_dict: Dict[str, torch.Tensor], cfg, device="cuda"):
        super().__init__()
        from .sparse import PackedSparseWeights, sparse_weight_blob

        load_ops()
        packed = PackedSparseWeights(state_dict, cfg, device)
        blob, icfg, fcfg = sparse_weight_blob(packed, cfg)
        self.register_buffer("blob", blob)
        self.icfg: List[int] = [int(x) for x in icfg]
        self.fcfg: List[float] = [float(x) for x in fcfg]

    def forward(self, pos: torch.Tensor, A: torch.Tensor, batch: torch.Tensor, edge_src: torch.Tensor,
                edge_dst: torch.Tensor, edge_shifts: torch.Tensor, cell: torch.Tensor, edge_vec: torch.Tensor,
                external_tensor: torch.Tensor) -> torch.Tensor:
        return torch.ops.fsctep.sparse_atom_energy(edge_vec, A, edge_src, edge_dst, self.blob, self.icfg, self.fcfg)


def _example_inputs(device, num_species: int):
    dev = torch.device(device)
    pos = torch.tensor([[0.0, 0.0, 0.0], [1.5, 0.3, -0.2], [0.4, 1.6, 0.5]], device=dev)
    A = (torch.arange(3, device=dev) % max(num_species, 1)).to(torch.int64)
    batch = torch.zeros(3, dtype=torch.int64, device=dev)
    src = torch.tensor([0, 1, 0, 2, 1, 2], device=dev)
    dst = torch.tensor([1, 0, 2, 0, 2, 1], device=dev)
    shifts = torch.zeros(6, 3, device=dev)
    cell = (torch.eye(3, device=dev) * 100.0).unsqueeze(0)
    edge_vec = pos[dst] - pos[src]
    ext = torch.empty(0, device=dev)
    return (pos, A, batch, src, dst, shifts, cell, edge_vec, ext)


def export_core(state_dict: Dict[str, torch.Tensor], cfg, path: str, device="cuda",
                element_types: List[str] | None = None) -> str:
    """Trace the core of an ``ICTDConfig`` (o3 or not) or ``SparseConfig`` model and save ``path``
    (core.pt) plus ``path + '.json'`` metadata."""
    from .sparse import SparseConfig

    if isinstance(cfg, SparseConfig):
        core, model = SparseCore(state_dict, cfg, device).eval(), "pure-cartesian-sparse"
    elif cfg.o3:
        core, model = ICTDO3Core(state_dict, cfg, device).eval(), "pure-cartesian-ictd-o3"
    else:
        core, model = ICTDCore(state_dict, cfg, device).eval(), "pure-cartesian-ictd"
    args = _example_inputs(device, cfg.max_atomvalue)
    field = model.endswith("o3")
    if field:
        args = args[:8] + (torch.zeros(3, device=args[0].device),)
    with torch.no_grad():
        traced = torch.jit.trace(core, args, check_trace=False)
    traced.save(path)
    meta = {"model": model, "backend": "fsctep_b200", "custom_ops_lib": os.path.basename(OPLIB),
            "cutoff": float(cfg.max_radius), "channels": int(cfg.channels), "lmax": int(cfg.lmax),
            "num_interaction": int(cfg.num_interaction), "max_atomvalue": int(cfg.max_atomvalue),
            "external_tensor_rank": 1 if field else None, "external_tensor_total_numel": 3 if field else 0,
            "num_fidelity_levels": 0, "export_reciprocal_source": False, "dtype": "float32"}
    if element_types is not None:
        meta["element_types"] = list(element_types)
    with open(path + ".json", "w") as f:
        json.dump(meta, f, indent=1)
    return path
