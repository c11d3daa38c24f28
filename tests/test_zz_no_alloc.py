"""Allocation-free CSR transpose (fsc_csr_transpose_static) against the workspace version.

The static entry point exists for callers that cannot allocate device memory, for example a
host program that gives all device memory to its own fixed pool or an FFI binding without a
device allocator: its scratch is a file-scope device array of the library instead of a caller
buffer.
This file is collected last so that a failure here never hides the other tests.
"""

import pytest
import torch

import gpu_util as U
from fsctep_b200 import _native as N
from fsctep_b200 import systems
from fsctep_b200.neighbors import build_graph

pytestmark = [pytest.mark.gpu, U.needs_gpu]


def _transpose_static(row_ptr, src, n):
    dev = src.device
    tr_ptr = torch.full((n + 1,), -7, dtype=torch.int32, device=dev)
    tr_eid = torch.full((max(src.numel(), 1),), -7, dtype=torch.int32, device=dev)
    N.check(N.lib().fsc_csr_transpose_static(N.ptr(row_ptr), N.ptr(src), n, src.numel(), N.ptr(tr_ptr),
                                             N.ptr(tr_eid), N.stream_ptr(dev)), "fsc_csr_transpose_static")
    return tr_ptr, tr_eid[:src.numel()]


def test_static_transpose_matches_workspace_version_twice():
    dev = torch.device("cuda")
    for seed, cells in ((31, (6, 6, 6)), (32, (5, 7, 4))):
        s = systems.diamond_crystal(n_cells=cells, seed=seed)
        g = build_graph(torch.tensor(s["pos"], device=dev), torch.tensor(s["cell"], device=dev), 5.0)
        tp, te = _transpose_static(g.row_ptr, g.src, g.num_atoms)
        torch.cuda.synchronize()
        assert torch.equal(tp, g.tr_ptr)
        assert torch.equal(te, g.tr_eid)


def test_static_transpose_rejects_oversized_input():
    dev = torch.device("cuda")
    row_ptr = torch.zeros(2, dtype=torch.int32, device=dev)
    src = torch.zeros(1, dtype=torch.int32, device=dev)
    st = N.lib().fsc_csr_transpose_static(N.ptr(row_ptr), N.ptr(src), 1 << 20, 1, N.ptr(row_ptr), N.ptr(src),
                                          N.stream_ptr(dev))
    assert st == 4
    assert b"at most" in N.lib().fsc_last_error()
