"""Product-side kernel tables vs the golden tables recorded from the reference."""

import numpy as np

import golden_io
from fsctep_b200 import tables as T


def test_product_tables_match_reference():
    z = golden_io.load("ictd_tables.npz")
    for L in range(5):
        np.testing.assert_allclose(T.harmonic_basis(L).numpy(), z[f"basis_{L}"], rtol=0, atol=1e-13)
        np.testing.assert_allclose(T.direction_projector(L).numpy(), z[f"dirproj_{L}"], rtol=0, atol=1e-12)
    paths = T.paths_full(2)
    for (l1, l2, l3) in paths:
        np.testing.assert_allclose(T.cg(l1, l2, l3).numpy(), z[f"L2_cg_{l1}{l2}{l3}"], rtol=0, atol=1e-13)
    np.testing.assert_allclose([T.p5_factor(l) for l in range(3)], z["L2_p5_factors"], atol=1e-14)


def test_kernel_table_direction_harmonics():
    """Y from the packed monomial table equals the reference direction harmonics."""
    z = golden_io.load("ictd_tables.npz")
    t = T.kernel_tables(2)
    yp = t[T.TAB_YPOLY:T.TAB_YPOLY + 90].reshape(10, 9)
    n = z["dir_n"]
    x, y, w = n[:, 0], n[:, 1], n[:, 2]
    mono = np.stack([np.ones_like(x), w, y, x, w * w, y * w, y * y, x * w, x * y, x * x], axis=1)
    Y = mono @ yp
    ref = np.concatenate([z["dir_Y_0"], z["dir_Y_1"], z["dir_Y_2"]], axis=1)
    np.testing.assert_allclose(Y, ref, atol=1e-12)


def test_kernel_table_coupling_reproduces_tp():
    """Yt[q] built from the 115x5 table equals the dense CG contraction for every path."""
    rng = np.random.default_rng(0)
    Yv = rng.normal(size=9)
    t = T.kernel_tables(2)
    cg2 = t[T.TAB_CG2:T.TAB_CG2 + 575].reshape(115, 5)
    for p, (l1, l2, l3) in enumerate(T.paths_full(2)):
        C = T.cg(l1, l2, l3).numpy()
        dense = np.einsum("mnk,n->mk", C, Yv[l2 * l2:l2 * l2 + 2 * l2 + 1])
        for m1 in range(2 * l1 + 1):
            for kk in range(2 * l3 + 1):
                q = T.QOFF[p] + m1 * (2 * l3 + 1) + kk
                got = sum(cg2[q, m] * Yv[l2 * l2 + m] for m in range(5) if l2 * l2 + m < 9)
                assert abs(got - dense[m1, kk]) < 1e-12
