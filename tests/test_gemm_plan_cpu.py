"""CPU check of the tensor-core GEMM plans: every GEMM shape the engines issue at the benchmark
widths keeps its tcgen05 accumulation chains at <= 24 MMAs (tensor-core accumulation rounds
toward zero, so longer chains bias long-K products), and the precise variant used for the
readout's Gram contraction at <= 12."""

import ctypes as C

import pytest

from fsctep_b200 import _native as N


def plan(K, Nc, precise=0):
    nt, chain = C.c_int(0), C.c_int(0)
    N.check(N.lib().fsc_gemm_tc_plan(K, Nc, precise, C.byref(nt), C.byref(chain)), "fsc_gemm_tc_plan")
    return nt.value, chain.value


def ictd_shapes(C_, nint, inv=32, hidden=(128, 128, 128), o3=False):
    np3, np1 = (3, 4, 4), (4, 4, 3)  # paths per l3 (forward) and per l1 (dx)
    out = []
    for l in range(3):
        out += [(np3[l] * C_, C_), (C_, np3[l] * C_), (np1[l] * C_, C_)]
    S = (nint - 1) * inv
    d0 = (4 if o3 else 3) * C_ * nint + S
    din = d0
    for h in hidden:
        out += [(din, h), (h, din)]
        din = h
    return out


def sparse_shapes(C_, lmax, nint, inv=32, hidden=(128, 128, 128)):
    npl = {2: (1, 2, 3), 3: (1, 2, 3, 4)}[lmax]  # paths per Lout (k0, max_rank_other 1)
    nC = C_ * nint
    S = (nint - 1) * inv
    shapes, precise = [], []
    for L in range(lmax + 1):
        K = npl[L] * 65 * C_
        shapes.append((K, C_))           # fc.4 after the aggregation
        shapes.append((C_, K))           # its transpose (dZ)
        precise.append((nC * (nC + 1) // 2, S))  # readout Gram contraction
        shapes.append((S, nC * nC))      # its gradient
    d0 = nint * C_ * (lmax + 1) + S
    din = d0
    for h in hidden:
        shapes += [(din, h), (h, din)]
        din = h
    return shapes, precise


@pytest.mark.parametrize("C_,nint,o3", [(32, 2, False), (64, 3, False), (64, 3, True)])
def test_ictd_gemm_chains_are_short(C_, nint, o3):
    for K, Nc in ictd_shapes(C_, nint, o3=o3):
        nt, chain = plan(K, Nc)
        assert chain <= 24, (K, Nc, nt, chain)


@pytest.mark.parametrize("C_,lmax", [(32, 2), (64, 2), (128, 3)])
def test_sparse_gemm_chains_are_short(C_, lmax):
    shapes, precise = sparse_shapes(C_, lmax, 3)
    for K, Nc in shapes:
        nt, chain = plan(K, Nc)
        assert chain <= 24, (K, Nc, nt, chain)
    for K, Nc in precise:
        nt, chain = plan(K, Nc, 1)
        assert chain <= 12, (K, Nc, nt, chain)


def test_wide_tiles_only_for_short_k():
    assert plan(128, 256) == (256, 24)
    nt, chain = plan(4096, 256)
    assert nt == 128 and chain <= 24


def test_plan_rejects_bad_sizes():
    nt, chain = C.c_int(0), C.c_int(0)
    assert N.lib().fsc_gemm_tc_plan(0, 64, 0, C.byref(nt), C.byref(chain)) != 0
