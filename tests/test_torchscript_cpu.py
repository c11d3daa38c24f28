"""core.pt op library on CPU: it loads without libpython, registers its schema and refuses CPU
tensors (the op has a CUDA kernel only)."""

import subprocess

import pytest
import torch

from fsctep_b200 import torchscript as TS


def test_op_library_registers_schema():
    TS.load_ops()
    op = torch.ops.fsctep.ictd_atom_energy
    schema = str(op.default._schema)
    assert schema.startswith("fsctep::ictd_atom_energy(Tensor edge_vec, Tensor species, Tensor edge_src, "
                             "Tensor edge_dst, Tensor blob, int[] icfg, float[] fcfg) -> Tensor"), schema


def test_op_library_has_no_python_dependency():
    out = subprocess.run(["ldd", TS.OPLIB], capture_output=True, text=True).stdout
    assert "libpython" not in out
    assert "libfsctep_b200.so" in out and "libtorch" in out


def test_cpu_tensors_are_rejected():
    TS.load_ops()
    z = torch.zeros(2, 3)
    with pytest.raises((RuntimeError, NotImplementedError)):
        torch.ops.fsctep.ictd_atom_energy(z, torch.zeros(2, dtype=torch.long), torch.zeros(2, dtype=torch.long),
                                          torch.zeros(2, dtype=torch.long), torch.zeros(4), [0] * 53, [5.0, 0.0])


def test_o3_and_sparse_ops_are_registered():
    TS.load_ops()
    o3 = str(torch.ops.fsctep.ictd_o3_atom_energy.default._schema)
    assert o3.startswith("fsctep::ictd_o3_atom_energy(Tensor edge_vec, Tensor species, Tensor edge_src, "
                         "Tensor edge_dst, Tensor field, Tensor blob, int[] icfg, float[] fcfg) -> Tensor"), o3
    sp = str(torch.ops.fsctep.sparse_atom_energy.default._schema)
    assert sp.startswith("fsctep::sparse_atom_energy(Tensor edge_vec, Tensor species, Tensor edge_src, "
                         "Tensor edge_dst, Tensor blob, int[] icfg, float[] fcfg) -> Tensor"), sp
