"""The native ASE calculator on the GPU against the reference's outputs.

``NativeCalculator`` replaces ``MyE3NNCalculator`` (``evaluation/calculator.py:89-172``): its
energy (plus the atomic reference energies), forces and stress (trainer convention, ASE Voigt
order) must match the reference fixtures.  The calculator needs only ``get_positions``,
``get_atomic_numbers``, ``get_cell`` and ``pbc`` of the atoms object (ASE itself is optional)."""

import numpy as np
import pytest
import torch

import golden_io
import gpu_util as U
from fsctep_b200.calculator import NativeCalculator, voigt
from fsctep_b200.models import PureCartesianICTDTransformerLayer

pytestmark = [pytest.mark.gpu, U.needs_gpu]


class _Atoms:
    def __init__(self, c):
        self._pos, self._num, self._cell = c["pos"], c["Z"], c["cell"][0]
        self.pbc = np.asarray(c["pbc"], dtype=bool)

    def get_positions(self):
        return self._pos

    def get_atomic_numbers(self):
        return self._num

    def get_cell(self):
        return self._cell


def _model(kind, tag):
    if kind == "ictd":
        cfg, sd, c = golden_io.model_case(tag)
        m = PureCartesianICTDTransformerLayer(max_embed_radius=5.0, main_max_radius=5.0, main_number_of_basis=8,
                                              hidden_dim_conv=int(cfg["channels"]),
                                              num_interaction=int(cfg["num_interaction"]),
                                              function_type_main=str(cfg["function_type"]),
                                              max_atomvalue=int(cfg["max_atomvalue"]))
    else:
        from test_models_cpu import _sparse_module

        cfg, sd, c = golden_io.sparse_case(tag)
        m = _sparse_module(cfg, device="cpu")
    m.load_state_dict({k: v.float() for k, v in sd.items()})
    return m.cuda(), c


@pytest.mark.parametrize("kind,tag", [("ictd", "b"), ("ictd", "c"), ("sparse", "a"), ("sparse", "d")])
def test_calculator_matches_reference(kind, tag):
    m, c = _model(kind, tag)
    e0 = {int(z): 0.25 * int(z) for z in np.unique(c["Z"])}
    calc = NativeCalculator(m, e0, "cuda", 5.0)
    atoms = _Atoms(c)
    calc.calculate(atoms, ("energy", "forces", "stress"))
    ref_e = float(c["ref64_energy"].sum()) + sum(e0[int(z)] for z in c["Z"])
    assert abs(calc.results["energy"] - ref_e) <= U.E_RTOL * abs(float(c["ref64_energy"].sum())) + 1e-9 * abs(ref_e)
    assert calc.results["free_energy"] == calc.results["energy"]
    assert U.rel_max(calc.results["forces"], c["ref64_forces"]) <= U.F_RTOL
    assert U.rel_max(calc.results["stress"], voigt(c["ref64_stress"][0])) <= U.S_RTOL
    # a second evaluation after moving one atom follows the positions
    atoms._pos = atoms._pos.copy()
    atoms._pos[0, 0] += 0.01
    calc.calculate(atoms, ("energy", "forces"))
    assert calc.results["energy"] != ref_e
