"""Host-side ICTD tables for the kernels (float64 on the CPU, computed once per lmax).

Mirrors the table construction of the reference (``models/ictd_irreps.py`` and
``models/ictd_fast.py``): harmonic basis as the Laplacian nullspace (SVD, rank threshold
1e-12) whitened under the isotropic-Gaussian Gram (eigh, floor 1e-14)
(``ictd_irreps.py:162-185``), Gram-weighted trace-chain projectors (``:229-254``), CG
tensors by polynomial product + projection (``:550-581``), "component" normalisation
(``:868-876``) and direction projectors ``G_l B_l`` (``:324-334``).  The same
linear-algebra calls in the same order make the basis identical to the reference's; the
golden tables recorded from the reference pin it (``tests/test_tables.py``).

``kernel_tables(lmax=2)`` packs what the sm_100a kernels read (layout in
``csrc/ictd_paths.cuh``): direction-harmonic polynomial coefficients, the conv2 coupling
table (115 x 5), the conv1 coupling table (9 x 5) and the product_5 0e factors.
"""

from __future__ import annotations

import math
from functools import lru_cache
from typing import Dict, List, Tuple

import numpy as np
import torch

F64 = torch.float64


def counts_list(L: int) -> List[Tuple[int, int, int]]:
    out = []
    for a in range(L + 1):
        for b in range(L - a + 1):
            out.append((a, b, L - a - b))
    return out


@lru_cache(maxsize=None)
def _gram(L: int) -> torch.Tensor:
    def mom(n):
        if n % 2:
            return 0.0
        r = 1
        for k in range(n - 1, 0, -2):
            r *= k
        return float(r)

    cl = counts_list(L)
    G = torch.zeros(len(cl), len(cl), dtype=F64)
    for i, (a, b, c) in enumerate(cl):
        for j, (d, e, f) in enumerate(cl):
            G[i, j] = mom(a + d) * mom(b + e) * mom(c + f)
    return G


def _laplacian(L: int) -> torch.Tensor:
    src, dst = counts_list(L), counts_list(L - 2)
    row = {t: i for i, t in enumerate(dst)}
    D = torch.zeros(len(dst), len(src), dtype=F64)
    for col, abc in enumerate(src):
        for ax in range(3):
            e = abc[ax]
            if e >= 2:
                t = list(abc)
                t[ax] -= 2
                D[row[tuple(t)], col] += float(e * (e - 1))
    return D


def _lift(l: int, k: int) -> torch.Tensor:
    src = counts_list(l)
    if k == 0:
        return torch.eye(len(src), dtype=F64)
    dst = counts_list(l + 2 * k)
    row = {t: i for i, t in enumerate(dst)}
    M = torch.zeros(len(dst), len(src), dtype=F64)
    terms = [(u, v, k - u - v, math.factorial(k) / (math.factorial(u) * math.factorial(v) * math.factorial(k - u - v)))
             for u in range(k + 1) for v in range(k - u + 1)]
    for col, (a, b, c) in enumerate(src):
        for u, v, w, coef in terms:
            M[row[(a + 2 * u, b + 2 * v, c + 2 * w)], col] += coef
    return M


@lru_cache(maxsize=None)
def harmonic_basis(L: int) -> torch.Tensor:
    if L == 0:
        return torch.ones(1, 1, dtype=F64)
    if L == 1:
        return torch.eye(3, dtype=F64)
    _, s, vh = torch.linalg.svd(_laplacian(L), full_matrices=True)
    rank = int((s > 1e-12).sum().item())
    B = vh[rank:].T.contiguous()
    ev, evec = torch.linalg.eigh(B.T @ _gram(L) @ B)
    W = evec @ torch.diag(torch.clamp(ev, min=1e-14).rsqrt()) @ evec.T
    return (B @ W).contiguous()


@lru_cache(maxsize=None)
def _projector(L: int, l: int) -> torch.Tensor:
    V = (_lift(l, (L - l) // 2) @ harmonic_basis(l)).contiguous()
    G = _gram(L)
    return torch.linalg.solve(V.T @ G @ V, V.T @ G).contiguous()


def field_l1_map() -> torch.Tensor:
    """(3, 3) M with t = M @ v: a Cartesian vector's ICTD l = 1 components (its monomial
    coefficients in ``counts_list(1)`` order projected with P_{1->1}), the embedding of a rank-1
    external tensor (pure_cartesian_ictd_layers.py:155-340)."""
    axis = [0 if a else (1 if b else 2) for (a, b, c) in counts_list(1)]
    sel = torch.zeros(3, 3, dtype=torch.float64)
    for d, ax in enumerate(axis):
        sel[d, ax] = 1.0
    return _projector(1, 1) @ sel


@lru_cache(maxsize=None)
def cg(l1: int, l2: int, l3: int) -> torch.Tensor:
    """Normalised ("component") coupling tensor C[m1, m2, m3]."""
    if not (abs(l1 - l2) <= l3 <= l1 + l2) or (l1 + l2 + l3) % 2:
        return torch.zeros(2 * l1 + 1, 2 * l2 + 1, 2 * l3 + 1, dtype=F64)
    c1, c2, cL = counts_list(l1), counts_list(l2), counts_list(l1 + l2)
    idx = {t: i for i, t in enumerate(cL)}
    M = torch.zeros(len(cL), len(c1) * len(c2), dtype=F64)
    for i, a in enumerate(c1):
        for j, b in enumerate(c2):
            M[idx[(a[0] + b[0], a[1] + b[1], a[2] + b[2])], i * len(c2) + j] = 1.0
    B1, B2 = harmonic_basis(l1), harmonic_basis(l2)
    outer = torch.einsum("im,jn->ijmn", B1, B2).reshape(B1.shape[0] * B2.shape[0], -1)
    C = (_projector(l1 + l2, l3) @ (M @ outer)).T.reshape(2 * l1 + 1, 2 * l2 + 1, 2 * l3 + 1).contiguous()
    fn = C.norm().item()
    if fn > 1e-30:
        C = C * (math.sqrt(2 * l3 + 1) / fn)
    return C


def paths_full(lmax: int) -> List[Tuple[int, int, int]]:
    """All (l1, l2, l3) of HarmonicFullyConnectedTensorProduct, reference order."""
    return [(l1, l2, l3) for l1 in range(lmax + 1) for l2 in range(lmax + 1)
            for l3 in range(abs(l1 - l2), min(l1 + l2, lmax) + 1) if (l1 + l2 + l3) % 2 == 0]


@lru_cache(maxsize=None)
def direction_projector(l: int) -> torch.Tensor:
    if l == 0:
        return torch.ones(1, 1, dtype=F64)
    return (_gram(l) @ harmonic_basis(l)).contiguous()


def p5_factor(l: int) -> float:
    return cg(l, l, 0)[0, 0, 0].item()


# ---- packed kernel tables (csrc/ictd_paths.cuh) -----------------------------------------------
NP, NK, NZ, NQ = 11, 9, 35, 115
TAB_YPOLY, TAB_CG2, TAB_CG1, TAB_P5, TAB_FLOATS = 0, 90, 665, 710, 720
QOFF = [0, 1, 4, 9, 18, 21, 36, 45, 70, 85, 90]


@lru_cache(maxsize=None)
def kernel_tables(lmax: int = 2) -> np.ndarray:
    if lmax != 2:
        raise NotImplementedError("the sm_100a ICTD kernels cover lmax = 2")
    t = np.zeros(TAB_FLOATS, dtype=np.float64)
    # direction harmonics: monomials 1 | z y x | zz yz yy xz xy xx  (counts_list order)
    mono_base = {0: 0, 1: 1, 2: 4}
    for l in range(3):
        P = direction_projector(l).numpy()
        cl = counts_list(l)
        for d, (a, b, c) in enumerate(cl):
            coef = math.factorial(l) / (math.factorial(a) * math.factorial(b) * math.factorial(c))
            for m in range(2 * l + 1):
                t[TAB_YPOLY + (mono_base[l] + d) * NK + l * l + m] = coef * P[d, m]
    paths = paths_full(2)
    for p, (l1, l2, l3) in enumerate(paths):
        C = cg(l1, l2, l3).numpy()
        for m1 in range(2 * l1 + 1):
            for kk in range(2 * l3 + 1):
                q = QOFF[p] + m1 * (2 * l3 + 1) + kk
                for m2 in range(2 * l2 + 1):
                    t[TAB_CG2 + 5 * q + m2] = C[m1, m2, kk]
    for l in range(3):
        C = cg(l, 0, l).numpy()
        for k in range(2 * l + 1):
            for m1 in range(2 * l + 1):
                t[TAB_CG1 + 5 * (l * l + k) + m1] = C[m1, 0, k]
    for l in range(3):
        t[TAB_P5 + l] = p5_factor(l)
    return t
