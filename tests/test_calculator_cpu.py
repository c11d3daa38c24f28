"""Host logic of the native ASE calculator on CPU, with a stand-in engine and graph builder
(the native engines and the cell list run on CUDA only)."""

import numpy as np
import pytest
import torch

from fsctep_b200.calculator import NativeCalculator, atomic_energy_offset, voigt


class _Atoms:
    def __init__(self, pos, numbers, cell, pbc):
        self._pos, self._num, self._cell, self.pbc = np.asarray(pos), np.asarray(numbers), np.asarray(cell), pbc

    def get_positions(self):
        return self._pos

    def get_atomic_numbers(self):
        return self._num

    def get_cell(self):
        return self._cell


class _Engine:
    """Records its inputs; energy = sum of x coordinates, forces = -1 along x, stress = given."""

    def __init__(self):
        self.calls = []

    def energy_forces(self, pos, species, batch, cell, g, want_stress=True, field=None):
        self.calls.append(dict(pos=pos, species=species, batch=batch, cell=cell, g=g, want_stress=want_stress,
                               field=field))
        f = torch.zeros_like(pos)
        f[:, 0] = -1.0
        out = {"energy": pos[:, 0].sum().reshape(1), "forces": f}
        if want_stress:
            out["stress"] = torch.arange(9, dtype=torch.float64).reshape(1, 3, 3)
        return out


def _graph_builder(log):
    def build(pos, cell, cutoff, pbc=(True, True, True), max_num_neighbors=None):
        assert max_num_neighbors == 100  # the reference builder's default cap
        log.append((cell.clone(), cutoff, pbc))
        return "graph"
    return build


def test_periodic_energy_forces_stress_and_offsets():
    eng, log = _Engine(), []
    calc = NativeCalculator(eng, {1: -0.5, 8: -2.0}, "cpu", 5.0, graph_builder=_graph_builder(log))
    atoms = _Atoms([[1.0, 0, 0], [2.0, 0, 0], [3.0, 0, 0]], [8, 1, 1], np.eye(3) * 9.0, np.array([True] * 3))
    calc.calculate(atoms)
    assert calc.results["energy"] == pytest.approx(6.0 - 3.0)
    assert calc.results["free_energy"] == calc.results["energy"]
    np.testing.assert_array_equal(calc.results["forces"][:, 0], [-1.0, -1.0, -1.0])
    np.testing.assert_array_equal(calc.results["stress"], [0.0, 4.0, 8.0, 5.0, 2.0, 1.0])
    cell, cutoff, pbc = log[0]
    np.testing.assert_array_equal(cell.numpy()[0], np.eye(3) * 9.0)
    assert cutoff == 5.0 and pbc == (True, True, True)
    call = eng.calls[0]
    assert call["want_stress"] and call["field"] is None
    assert call["species"].tolist() == [8, 1, 1] and call["batch"].tolist() == [0, 0, 0]


def test_molecule_uses_the_reference_standin_cell_and_no_stress():
    eng, log = _Engine(), []
    calc = NativeCalculator(eng, {6: 1.0}, "cpu", 4.0, graph_builder=_graph_builder(log),
                            external_tensor=torch.tensor([0.1, 0.2, 0.3]))
    calc.calculate(_Atoms([[0.5, 0, 0], [1.5, 0, 0]], [6, 6], np.zeros((3, 3)), np.array([False] * 3)))
    assert "stress" not in calc.results
    np.testing.assert_array_equal(log[0][0].numpy()[0], np.eye(3) * 100.0)
    assert log[0][2] == (False, False, False)
    assert not eng.calls[0]["want_stress"]
    np.testing.assert_allclose(eng.calls[0]["field"].numpy(), [[0.1, 0.2, 0.3]], rtol=1e-6)
    assert calc.results["energy"] == pytest.approx(2.0 + 2.0)


def test_missing_atomic_energy_and_unsupported_options():
    with pytest.raises(KeyError):
        atomic_energy_offset(np.array([1, 8, 26]), {1: 0.0, 8: 0.0})
    with pytest.raises(NotImplementedError):
        NativeCalculator(_Engine(), {}, "cpu", 5.0, fidelity_id=1)
    with pytest.raises(NotImplementedError):
        NativeCalculator(_Engine(), {}, "cpu", 5.0, return_physical_tensors=True)


def test_native_path_refuses_cpu_devices():
    calc = NativeCalculator(_Engine(), {1: 0.0}, "cpu", 5.0)
    with pytest.raises(RuntimeError, match="CUDA"):
        calc.calculate(_Atoms([[0.0, 0, 0]], [1], np.eye(3) * 10, np.array([True] * 3)))


def test_voigt_order():
    s = np.arange(9.0).reshape(3, 3)
    np.testing.assert_array_equal(voigt(s), [0, 4, 8, 5, 2, 1])
