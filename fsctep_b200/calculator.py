"""ASE calculator over the native engines.

Drop-in for ``MyE3NNCalculator`` (``evaluation/calculator.py:40-172``) with the drop-in models of
:mod:`fsctep_b200.models`: same constructor arguments and ``results``, but ``calculate`` calls the
engine's fused energy + forces (+ stress) on the GPU cell-list neighbour list instead of
``radius_graph_pbc_gpu`` (``utils/graph_utils.py:192-258``) followed by a model forward and an
autograd replay (``calculator.py:120-159``).

* Atomic reference energies are added as the reference does (``map_tensor_values``,
  ``utils/tensor_utils.py:36-76``): every atomic number of the system must be a key, else
  ``KeyError``.
* A system with no periodic axis gets the reference's stand-in cell (identity x 100 A) and no
  periodicity; with any periodic axis the atoms' cell and pbc flags are used.
* ``results["stress"]`` (periodic systems) is (1/V) dE/d(strain), the trainer's convention
  (``training/trainer.py:1213-1310``), in ASE's Voigt order (xx, yy, zz, yz, xz, xy).
* ``external_tensor`` (the o3 model's rank-1 field) is passed to the engine as the graph's field.

Without ASE installed the class still works with any object offering ``get_positions``,
``get_atomic_numbers``, ``get_cell`` and ``pbc`` (the ``atoms`` argument of ``calculate``).
There is no CPU path: the engines and the neighbour builder run on CUDA devices only.
"""

from __future__ import annotations

from typing import Any, Callable, Dict, Optional

import numpy as np
import torch

try:  # ASE is optional
    from ase.calculators.calculator import Calculator as _Base
    from ase.calculators.calculator import all_changes as _ALL_CHANGES
except ImportError:  # pragma: no cover - exercised where ASE is absent
    _ALL_CHANGES = ("positions", "numbers", "cell", "pbc")

    class _Base:
        """Minimal stand-in for ``ase.calculators.calculator.Calculator``."""

        implemented_properties: list = []

        def __init__(self, **kwargs):
            self.atoms = None
            self.results: Dict[str, Any] = {}
            self.parameters = dict(kwargs)

        def calculate(self, atoms=None, properties=("energy",), system_changes=_ALL_CHANGES):
            if atoms is not None:
                self.atoms = atoms
            self.results = {}

        def get_property(self, name, atoms=None):
            self.calculate(atoms, (name,))
            return self.results[name]

        def get_potential_energy(self, atoms=None):
            return self.get_property("energy", atoms)

        def get_forces(self, atoms=None):
            return self.get_property("forces", atoms)

        def get_stress(self, atoms=None):
            return self.get_property("stress", atoms)

STANDIN_CELL = 100.0  # non-periodic systems: identity x 100 A (calculator.py:113-118)


def atomic_energy_offset(numbers: np.ndarray, atomic_energies: Dict[int, float]) -> float:
    """Sum of the atoms' reference energies; every atomic number must be a key."""
    numbers = np.asarray(numbers, dtype=np.int64)
    missing = sorted(set(numbers.tolist()) - set(int(k) for k in atomic_energies))
    if missing:
        raise KeyError(f"atomic energies missing for atomic numbers {missing}: provide atomic_energies_dict "
                       "entries that cover all elements in the system")
    return float(sum(float(atomic_energies[int(z)]) for z in numbers))


def voigt(stress: np.ndarray) -> np.ndarray:
    """3x3 -> ASE Voigt order (xx, yy, zz, yz, xz, xy)."""
    s = np.asarray(stress, dtype=np.float64).reshape(3, 3)
    return np.array([s[0, 0], s[1, 1], s[2, 2], s[1, 2], s[0, 2], s[0, 1]])


class NativeCalculator(_Base):
    """Energy, forces and (periodic systems) stress from a drop-in model's native engine.

    Args (as ``MyE3NNCalculator``):
        model: a drop-in model of :mod:`fsctep_b200.models` (or an engine with ``energy_forces``).
        atomic_energies_dict: atomic number -> E0.
        device: CUDA device.
        max_radius: neighbour cutoff (A).
        external_tensor: the o3 model's rank-1 field, shape (3,) or (1, 3), or None.
        fidelity_id, return_physical_tensors: not covered by the native engines (must be None / False).
        graph_builder: ``(pos, cell, cutoff, pbc=...) -> GraphCSR``; default the GPU cell list.
    """

    implemented_properties = ["energy", "free_energy", "forces", "stress"]

    def __init__(self, model, atomic_energies_dict: Dict[int, float], device, max_radius: float,
                 external_tensor: Optional[torch.Tensor] = None, fidelity_id: Optional[int] = None,
                 return_physical_tensors: bool = False, graph_builder: Optional[Callable] = None,
                 max_num_neighbors: Optional[int] = 100, **kwargs: Any):
        if fidelity_id is not None or return_physical_tensors:
            raise NotImplementedError("fsctep_b200 calculator: multi-fidelity and physical-tensor outputs are "
                                      "not covered by the native engines")
        _Base.__init__(self, **kwargs)
        self.model = model
        self.device = torch.device(device)
        self.max_radius = float(max_radius)
        self.atomic_energies = {int(k): float(v) for k, v in atomic_energies_dict.items()}
        self.external_tensor = external_tensor
        # the reference's graph builder caps each source at 100 candidates per image shift
        # (radius_graph_pbc_gpu's default, utils/graph_utils.py:192); None lifts the cap
        self.max_num_neighbors = max_num_neighbors
        self.native = graph_builder is None  # the GPU cell list and a native engine
        if graph_builder is None:
            from .neighbors import build_graph as graph_builder
        self.graph_builder = graph_builder

    def _engine(self):
        if hasattr(self.model, "_ensure_engine"):
            return self.model._ensure_engine(self.device)
        return self.model

    def calculate(self, atoms=None, properties=("energy", "forces"), system_changes=_ALL_CHANGES):
        _Base.calculate(self, atoms, properties, system_changes)
        atoms = self.atoms
        if self.native and self.device.type != "cuda":
            raise RuntimeError("fsctep_b200 runs on CUDA devices only (no CPU path)")
        numbers = np.asarray(atoms.get_atomic_numbers(), dtype=np.int64)
        pbc = tuple(bool(p) for p in np.broadcast_to(np.asarray(atoms.pbc), (3,)))
        periodic = any(pbc)
        if periodic:
            cell = np.asarray(getattr(atoms.get_cell(), "array", atoms.get_cell()), dtype=np.float64)
        else:
            cell = np.eye(3) * STANDIN_CELL
        e0 = atomic_energy_offset(numbers, self.atomic_energies)
        dev = self.device
        pos = torch.tensor(np.asarray(atoms.get_positions(), dtype=np.float64), device=dev)
        cell_t = torch.tensor(cell, device=dev).reshape(1, 3, 3)
        species = torch.tensor(numbers, device=dev, dtype=torch.int32)
        batch = torch.zeros(len(numbers), device=dev, dtype=torch.int32)
        graph = self.graph_builder(pos, cell_t, self.max_radius, pbc=pbc, max_num_neighbors=self.max_num_neighbors)
        kwargs = {}
        if self.external_tensor is not None:
            kwargs["field"] = torch.as_tensor(self.external_tensor, device=dev).reshape(1, 3)
        out = self._engine().energy_forces(pos, species, batch, cell_t, graph, want_stress=periodic, **kwargs)
        energy = float(out["energy"].double().sum().item()) + e0
        self.results["energy"] = energy
        self.results["free_energy"] = energy
        self.results["forces"] = out["forces"].double().cpu().numpy()
        if periodic:
            self.results["stress"] = voigt(out["stress"][0].double().cpu().numpy())
