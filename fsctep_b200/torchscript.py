"""core.pt export: the pure-cartesian-ictd model as a traced TorchScript module whose only
compute is the ``fsctep::ictd_atom_energy`` custom op (torch_ops/ictd_op.cpp).

Signature and outputs follow the reference's traced core (``_TorchScriptEdgeVecCore``,
interfaces/lammps_mliap.py:372-420, exported by cli/export_libtorch_core.py):
``forward(pos, A, batch, edge_src, edge_dst, edge_shifts, cell, edge_vec, external_tensor)
-> atom_energy (N, 1)``, differentiable with respect to ``edge_vec`` (the LAMMPS engine,
mff_torch_engine.cpp:459-569, takes ``autograd::grad`` of the local energy through it).  Load the
op library before ``torch.jit.load`` (LAMMPS: ``MFF_CUSTOM_OPS_LIB=<op library path>``).
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


def export_core(state_dict: Dict[str, torch.Tensor], cfg: ICTDConfig, path: str, device="cuda",
                element_types: List[str] | None = None) -> str:
    """Trace the core and save ``path`` (core.pt) plus ``path + '.json'`` metadata."""
    core = ICTDCore(state_dict, cfg, device).eval()
    with torch.no_grad():
        traced = torch.jit.trace(core, _example_inputs(device, cfg.max_atomvalue), check_trace=False)
    traced.save(path)
    meta = {"model": "pure-cartesian-ictd", "backend": "fsctep_b200", "custom_ops_lib": os.path.basename(OPLIB),
            "cutoff": float(cfg.max_radius), "channels": int(cfg.channels), "lmax": int(cfg.lmax),
            "num_interaction": int(cfg.num_interaction), "max_atomvalue": int(cfg.max_atomvalue),
            "external_tensor_rank": None, "external_tensor_total_numel": 0, "num_fidelity_levels": 0,
            "export_reciprocal_source": False, "dtype": "float32"}
    if element_types is not None:
        meta["element_types"] = list(element_types)
    with open(path + ".json", "w") as f:
        json.dump(meta, f, indent=1)
    return path
