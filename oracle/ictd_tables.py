"""ICTD host tables, restated on the CPU in float64 (test infrastructure only).

Follows ``models/ictd_irreps.py`` and ``models/ictd_fast.py`` of the reference:

* monomial orbits of degree L: ``ictd_fast.py:41-48`` (``_counts_list``);
* isotropic-Gaussian Gram matrix on Sym^L: ``ictd_irreps.py:143-159``;
* Laplacian Sym^L -> Sym^{L-2}: ``ictd_fast.py:83-114``;
* r^{2k} lift Sym^l -> Sym^{l+2k}: ``ictd_fast.py:240-266``;
* harmonic basis = Laplacian nullspace (SVD) + Gram whitening (eigh):
  ``ictd_irreps.py:162-185``;
* trace-chain projectors (Gram-weighted least squares): ``ictd_irreps.py:229-254``;
* polynomial product matrix and CG tensor: ``ictd_irreps.py:516-581``;
* path enumeration, "component" normalisation and (l1,l2) group packing of U:
  ``ictd_irreps.py:801-934``;
* direction harmonics ``Y_l(n) = (multinomial * n^abc) @ (G_l B_l)``:
  ``ictd_irreps.py:304-402``.

The harmonic basis is unique only up to an orthogonal transform, so the same
linear-algebra calls (``torch.linalg.svd`` with ``full_matrices=True``, rank
threshold 1e-12, ``torch.linalg.eigh`` whitening with eigenvalue floor 1e-14)
are used in the same order as the reference; the golden tables recorded from
the reference pin the result.
"""

from __future__ import annotations

import math
from functools import lru_cache
from typing import Dict, List, Tuple

import torch

F64 = torch.float64


def counts_list(L: int) -> List[Tuple[int, int, int]]:
    """(a, b, c) exponents of x^a y^b z^c with a+b+c=L (a outer, b inner)."""
    return [(a, b, L - a - b) for a in range(L + 1) for b in range(L - a + 1)]


def sym_dim(L: int) -> int:
    return (L + 1) * (L + 2) // 2


def _gauss_moment(n: int) -> float:
    if n % 2:
        return 0.0
    v = 1
    for k in range(n - 1, 0, -2):
        v *= k
    return float(v)


@lru_cache(maxsize=None)
def gram_gaussian(L: int) -> torch.Tensor:
    cl = counts_list(L)
    G = torch.zeros(len(cl), len(cl), dtype=F64)
    for i, (a, b, c) in enumerate(cl):
        for j, (d, e, f) in enumerate(cl):
            G[i, j] = _gauss_moment(a + d) * _gauss_moment(b + e) * _gauss_moment(c + f)
    return G


def laplacian_matrix(L: int) -> torch.Tensor:
    src, dst = counts_list(L), counts_list(L - 2)
    row_of = {t: i for i, t in enumerate(dst)}
    D = torch.zeros(len(dst), len(src), dtype=F64)
    for col, (a, b, c) in enumerate(src):
        for axis, e in enumerate((a, b, c)):
            if e >= 2:
                t = [a, b, c]
                t[axis] -= 2
                D[row_of[tuple(t)], col] += float(e * (e - 1))
    return D


def r2k_lift(l: int, k: int) -> torch.Tensor:
    src = counts_list(l)
    if k == 0:
        return torch.eye(len(src), dtype=F64)
    dst = counts_list(l + 2 * k)
    row_of = {t: i for i, t in enumerate(dst)}
    M = torch.zeros(len(dst), len(src), dtype=F64)
    terms = []
    for u in range(k + 1):
        for v in range(k - u + 1):
            w = k - u - v
            terms.append((u, v, w, math.factorial(k) / (math.factorial(u) * math.factorial(v) * math.factorial(w))))
    for col, (a, b, c) in enumerate(src):
        for u, v, w, coef in terms:
            M[row_of[(a + 2 * u, b + 2 * v, c + 2 * w)], col] += coef
    return M


@lru_cache(maxsize=None)
def harmonic_basis(L: int) -> torch.Tensor:
    """(Dsym(L), 2L+1) G-orthonormal basis of the harmonic polynomials of degree L."""
    if L == 0:
        return torch.ones(1, 1, dtype=F64)
    if L == 1:
        return torch.eye(3, dtype=F64)
    _, s, vh = torch.linalg.svd(laplacian_matrix(L), full_matrices=True)
    rank = int((s > 1e-12).sum().item())
    B = vh[rank:].T.contiguous()
    G = gram_gaussian(L)
    ev, evec = torch.linalg.eigh(B.T @ G @ B)
    ev = torch.clamp(ev, min=1e-14)
    W = evec @ torch.diag(ev.rsqrt()) @ evec.T
    return (B @ W).contiguous()


@lru_cache(maxsize=None)
def projector(L: int, l: int) -> torch.Tensor:
    """P_{L->l}: (2l+1, Dsym(L)) Gram-weighted projection onto r^{L-l} Harm^l."""
    k = (L - l) // 2
    V = (r2k_lift(l, k) @ harmonic_basis(l)).contiguous()
    GL = gram_gaussian(L)
    return torch.linalg.solve(V.T @ GL @ V, V.T @ GL).contiguous()


def poly_mult_matrix(l1: int, l2: int) -> torch.Tensor:
    c1, c2, cL = counts_list(l1), counts_list(l2), counts_list(l1 + l2)
    idx = {t: i for i, t in enumerate(cL)}
    M = torch.zeros(len(cL), len(c1) * len(c2), dtype=F64)
    for i, (a, b, c) in enumerate(c1):
        for j, (d, e, f) in enumerate(c2):
            M[idx[(a + d, b + e, c + f)], i * len(c2) + j] = 1.0
    return M


@lru_cache(maxsize=None)
def cg_tensor(l1: int, l2: int, l3: int) -> torch.Tensor:
    """Raw coupling tensor C[m1, m2, m3] in the ICTD harmonic basis."""
    if not (abs(l1 - l2) <= l3 <= l1 + l2) or (l1 + l2 + l3) % 2:
        return torch.zeros(2 * l1 + 1, 2 * l2 + 1, 2 * l3 + 1, dtype=F64)
    L = l1 + l2
    B1, B2 = harmonic_basis(l1), harmonic_basis(l2)
    outer = torch.einsum("im,jn->ijmn", B1, B2).reshape(B1.shape[0] * B2.shape[0], -1)
    c3 = projector(L, l3) @ (poly_mult_matrix(l1, l2) @ outer)
    return c3.T.reshape(2 * l1 + 1, 2 * l2 + 1, 2 * l3 + 1).contiguous()


def normalized_cg(l1: int, l2: int, l3: int, normalization: str = "component") -> torch.Tensor:
    C = cg_tensor(l1, l2, l3)
    fn = C.norm().item()
    if normalization == "component" and fn > 1e-30:
        C = C * (math.sqrt(2 * l3 + 1) / fn)
    elif normalization == "norm" and fn > 1e-30:
        C = C * (1.0 / fn)
    return C


def tp_paths(lmax: int, path_policy: str = "full", max_rank_other=None, allowed_paths=None):
    """Path list of HarmonicFullyConnectedTensorProduct (ictd_irreps.py:801-821)."""
    allp = []
    for l1 in range(lmax + 1):
        for l2 in range(lmax + 1):
            for l3 in range(abs(l1 - l2), min(l1 + l2, lmax) + 1):
                if (l1 + l2 + l3) % 2 == 0:
                    allp.append((l1, l2, l3))
    if allowed_paths is not None:
        keep = set(tuple(p) for p in allowed_paths)
        return [p for p in allp if p in keep]
    if path_policy == "full":
        return allp
    if path_policy == "max_rank_other":
        if max_rank_other is None:
            raise ValueError("path_policy='max_rank_other' requires max_rank_other")
        return [p for p in allp if min(p[0], p[1]) <= int(max_rank_other)]
    raise ValueError(f"Unknown path_policy={path_policy!r}")


def tp_groups(paths):
    """(l1,l2) groups with (p_idx, l3, start, end) segments (ictd_irreps.py:854-877)."""
    tmp: Dict[Tuple[int, int], list] = {}
    for p, (l1, l2, l3) in enumerate(paths):
        tmp.setdefault((l1, l2), []).append((p, l3))
    out = []
    for (l1, l2), items in sorted(tmp.items()):
        segs, s = [], 0
        for p, l3 in items:
            segs.append((p, l3, s, s + 2 * l3 + 1))
            s += 2 * l3 + 1
        out.append({"l1": l1, "l2": l2, "segments": segs, "k_total": s})
    return out


def group_U(paths, groups, normalization: str = "component") -> List[torch.Tensor]:
    """U_g (m1*m2, K_total) per group (ictd_irreps.py:882-934)."""
    Us = []
    for g in groups:
        m1, m2 = 2 * g["l1"] + 1, 2 * g["l2"] + 1
        U = torch.zeros(m1 * m2, g["k_total"], dtype=F64)
        for p, l3, s, e in g["segments"]:
            l1, l2, _ = paths[p]
            U[:, s:e] = normalized_cg(l1, l2, l3, normalization).reshape(m1 * m2, e - s)
        Us.append(U)
    return Us


@lru_cache(maxsize=None)
def direction_projector(l: int) -> torch.Tensor:
    """G_l @ B_l, (Dsym(l), 2l+1) (ictd_irreps.py:324-334)."""
    if l == 0:
        return torch.ones(1, 1, dtype=F64)
    return (gram_gaussian(l) @ harmonic_basis(l)).contiguous()


def monomial_coefs(l: int) -> torch.Tensor:
    if l == 0:
        return torch.ones(1, dtype=F64)
    return torch.tensor([math.factorial(l) / (math.factorial(a) * math.factorial(b) * math.factorial(c))
                         for (a, b, c) in counts_list(l)], dtype=F64)


def direction_harmonics(n: torch.Tensor, l: int) -> torch.Tensor:
    """Y_l(n), (..., 2l+1) (ictd_irreps.py:371-402); integer power tables as in :337-348."""
    if l == 0:
        return torch.ones(*n.shape[:-1], 1, dtype=n.dtype)
    exps = torch.tensor(counts_list(l), dtype=torch.int64)
    pw = []
    for axis in range(3):
        cur = torch.ones_like(n[..., axis])
        col = [cur]
        for _ in range(l):
            cur = cur * n[..., axis]
            col.append(cur)
        pw.append(torch.stack(col, dim=-1))
    t = pw[0][..., exps[:, 0]] * pw[1][..., exps[:, 1]] * pw[2][..., exps[:, 2]]
    t = t * monomial_coefs(l).to(n.dtype)
    return t @ direction_projector(l).to(n.dtype)
