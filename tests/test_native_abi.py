"""CPU-side checks of the C ABI: the library loads and exports every declared entry point."""

import os
import re

import pytest

from fsctep_b200 import _native as N

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _declared():
    src = open(os.path.join(ROOT, "include", "fsctep_b200.h")).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    return sorted(set(re.findall(r"\b(fsc_[a-z0-9_]+)\s*\(", src)))


def test_header_and_binding_agree():
    assert _declared() == N.exported_symbols()


def test_library_exports_every_declared_symbol():
    lib = N.lib()
    for name in _declared():
        assert hasattr(lib, name), name


def test_library_queries_without_gpu():
    lib = N.lib()
    assert lib.fsc_has_cuda() == 1
    assert lib.fsc_ictd_tables_floats() == 720
    assert lib.fsc_neighbor_workspace_bytes(1000, 0) > 0


def test_unsupported_config_reports_zero_workspace():
    import ctypes
    cfg = N.IctdConfig(channels=48, lmax=2, num_interaction=3, number_of_basis=8, basis_kind=0, max_radius=5.0,
                       num_species=10, output_size=8, invariant_channels=32, n_hidden=1, n_out=17)
    cfg.hidden[0] = 128
    assert N.lib().fsc_ictd_workspace_bytes(ctypes.byref(cfg), 10, 10) == 0


def test_argument_errors_are_reported_not_raised_in_c():
    # a bad dtype is rejected before any device work
    st = N.lib().fsc_project_bucket_forward(7, None, None, None, None, 1, 1, 1, 1, 1, 1, 1, None)
    assert st == 1
    assert b"dtype" in N.lib().fsc_last_error()


def test_struct_layouts_agree_with_the_c_header(tmp_path):
    """sizeof and field offsets of every ABI struct, as compiled from include/fsctep_b200.h by the C
    compiler, equal the ctypes mirrors the host side passes by pointer."""
    import shutil
    import subprocess

    cc = shutil.which("gcc") or shutil.which("cc")
    if cc is None:
        pytest.skip("no C compiler")
    structs = {"fsc_ictd_config": N.IctdConfig, "fsc_ictd_weights": N.IctdWeights,
               "fsc_sparse_config": N.SparseConfig, "fsc_sparse_weights": N.SparseWeights,
               "fsc_graph": N.Graph, "fsc_ictd_outputs": N.IctdOutputs}
    lines = ['#include <stdio.h>', '#include <stddef.h>', '#include "fsctep_b200.h"', "int main(void) {"]
    for cname, py in structs.items():
        lines.append(f'  printf("{cname} sizeof %zu\\n", sizeof({cname}));')
        for field, _ in py._fields_:
            lines.append(f'  printf("{cname} {field} %zu\\n", offsetof({cname}, {field}));')
    lines += ["  return 0;", "}"]
    src = tmp_path / "layout.c"
    src.write_text("\n".join(lines))
    exe = tmp_path / "layout"
    subprocess.run([cc, "-std=c99", "-I", os.path.join(ROOT, "include"), str(src), "-o", str(exe)], check=True)
    out = subprocess.run([str(exe)], check=True, capture_output=True, text=True).stdout.split("\n")
    got = {(a, b): int(c) for a, b, c in (ln.split() for ln in out if ln)}
    for cname, py in structs.items():
        assert got[(cname, "sizeof")] == __import__("ctypes").sizeof(py), cname
        for field, _ in py._fields_:
            assert got[(cname, field)] == getattr(py, field).offset, (cname, field)


def test_static_transpose_capacity_checked_before_device_work():
    """The allocation-free transpose rejects sizes beyond its static scratch with a capacity error
    before any device call; at its stated limits the capacity check passes (on a machine without
    a GPU the call then fails on the device query instead)."""
    L = N.lib()
    st = L.fsc_csr_transpose_static(None, None, 262144 + 1, 10, None, None, None)
    assert st == 4 and b"at most" in L.fsc_last_error()
    st = L.fsc_csr_transpose_static(None, None, 10, 4194304 + 1, None, None, None)
    assert st == 4
    st = L.fsc_csr_transpose_static(None, None, 262144, 4194304, None, None, None)
    assert st != 4, L.fsc_last_error()
