"""`_C_ictd_tp` operator family through the C ABI vs the reference einsum definitions."""

import numpy as np
import pytest
import torch

import golden_io
import gpu_util as U
from fsctep_b200 import _C_ictd_tp as ext

pytestmark = [pytest.mark.gpu, U.needs_gpu]

TOL = {torch.float32: (1e-5, 1e-6), torch.float64: (1e-10, 1e-12)}


def _ref_project(a, b, u, P):
    B, I, m1 = a.shape
    _, J, m2 = b.shape
    pk = u.shape[1]
    y = torch.einsum("bim,bjn,mnp->bijp", a, b, u.view(m1, m2, pk))
    return y.reshape(B, I * J, P, pk // P).permute(0, 2, 3, 1).contiguous()


def _ref_mix(y, w, g):
    return (torch.einsum("bpkq,poq->bpok", y, w) * g[:, :, None, None]).sum(1)


def test_golden_fixture_ops():
    z = golden_io.load("tp_ops.npz")
    t = {k: torch.tensor(z[k], device="cuda") for k in z.files}
    P = t["w"].shape[0]
    torch.testing.assert_close(ext.project_bucket_forward(t["a"], t["b"], t["U"], P), t["y"], rtol=1e-10, atol=1e-12)
    torch.testing.assert_close(ext.project_bucket_transpose_a(t["gy"], t["b"], t["U"]), t["ga"], rtol=1e-10, atol=1e-12)
    torch.testing.assert_close(ext.project_bucket_transpose_b(t["gy"], t["a"], t["U"]), t["gb"], rtol=1e-10, atol=1e-12)
    torch.testing.assert_close(ext.project_bucket_transpose_u(t["gy"], t["a"], t["b"]), t["gu"], rtol=1e-10, atol=1e-12)
    torch.testing.assert_close(ext.mix_bucket_forward(t["y"], t["w"], t["gates"]), t["mo"], rtol=1e-10, atol=1e-12)
    torch.testing.assert_close(ext.mix_bucket_transpose_y(t["go"], t["w"], t["gates"]), t["my"], rtol=1e-10, atol=1e-12)
    torch.testing.assert_close(ext.mix_bucket_transpose_w(t["go"], t["y"], t["gates"]), t["mw"], rtol=1e-10, atol=1e-12)
    torch.testing.assert_close(ext.mix_bucket_transpose_g(t["go"], t["y"], t["w"]), t["mg"], rtol=1e-10, atol=1e-12)


@pytest.mark.parametrize("dtype", [torch.float32, torch.float64])
@pytest.mark.parametrize("J", [1, 2])
def test_projection_family_random(dtype, J):
    rtol, atol = TOL[dtype]
    g = torch.Generator().manual_seed(11 + J)
    B, I, m1, m2, P, K, O = 5, 3, 5, 3, 3, 5, 4
    a = torch.randn(B, I, m1, generator=g, dtype=dtype).cuda()
    b = torch.randn(B, J, m2, generator=g, dtype=dtype).cuda()
    u = torch.randn(m1 * m2, P * K, generator=g, dtype=dtype).cuda()
    w = torch.randn(P, O, I * J, generator=g, dtype=dtype).cuda()
    gates = torch.randn(B, P, generator=g, dtype=dtype).cuda()
    y = _ref_project(a, b, u, P)
    torch.testing.assert_close(ext.project_bucket_forward(a, b, u, P), y, rtol=rtol, atol=atol)
    torch.testing.assert_close(ext.bucketed_tp_forward(a, b, u, w, gates), _ref_mix(y, w, gates),
                               rtol=rtol * 10, atol=atol * 10)
    a_, b_, u_ = (x.clone().requires_grad_(True) for x in (a, b, u))
    gy = torch.randn(y.shape, generator=g, dtype=dtype).cuda()
    ga, gb, gu = torch.autograd.grad(_ref_project(a_, b_, u_, P), (a_, b_, u_), gy)
    torch.testing.assert_close(ext.project_bucket_transpose_a(gy, b, u), ga, rtol=rtol, atol=atol)
    torch.testing.assert_close(ext.project_bucket_transpose_b(gy, a, u), gb, rtol=rtol, atol=atol)
    torch.testing.assert_close(ext.project_bucket_transpose_u(gy, a, b), gu, rtol=rtol, atol=atol)


@pytest.mark.parametrize("dtype", [torch.float32, torch.float64])
def test_double_backward_family(dtype):
    rtol, atol = (5e-5, 5e-6) if dtype == torch.float32 else (1e-10, 1e-12)
    gen = torch.Generator().manual_seed(500)
    B, I, m1, m2, P, K, O = 3, 2, 3, 3, 2, 3, 4
    mk = lambda *s: torch.randn(*s, generator=gen, dtype=dtype).cuda()  # noqa: E731
    h, a, b, u = mk(B, P, K, I), mk(B, I, m1), mk(B, 1, m2), mk(m1 * m2, P * K)
    gga, ggb, ggu = mk(B, I, m1), mk(B, 1, m2), mk(m1 * m2, P * K)
    PF = lambda a_, b_, u_: _ref_project(a_, b_, u_, P)  # noqa: E731
    torch.testing.assert_close(ext.project_dbl_bwd_grad_h(a, gga, b, ggb, u, ggu, P),
                               PF(gga, b, u) + PF(a, ggb, u) + PF(a, b, ggu), rtol=rtol, atol=atol)
    y, w, gates, go = mk(B, P, K, I), mk(P, O, I), mk(B, P), mk(B, O, K)
    ggy, ggw, ggg = mk(B, P, K, I), mk(P, O, I), mk(B, P)
    torch.testing.assert_close(ext.mix_dbl_bwd_grad_g_out(y, ggy, w, ggw, gates, ggg),
                               _ref_mix(ggy, w, gates) + _ref_mix(y, ggw, gates) + _ref_mix(y, w, ggg),
                               rtol=rtol, atol=atol)
    # adjoint identities: <PAT(h,b,u), x> = <h, PF(x,b,u)>
    x = mk(B, I, m1)
    lhs = (ext.project_dbl_bwd_grad_a(h, b, ggb, u, ggu) * x).sum()
    rhs = (h * (PF(x, ggb, u) + PF(x, b, ggu))).sum()
    torch.testing.assert_close(lhs, rhs, rtol=rtol * 10, atol=atol * 10)
    xb = mk(B, 1, m2)
    lhs = (ext.project_dbl_bwd_grad_b(h, a, gga, u, ggu) * xb).sum()
    rhs = (h * (PF(gga, xb, u) + PF(a, xb, ggu))).sum()
    torch.testing.assert_close(lhs, rhs, rtol=rtol * 10, atol=atol * 10)
    xu = mk(m1 * m2, P * K)
    lhs = (ext.project_dbl_bwd_grad_u(h, a, gga, b, ggb) * xu).sum()
    rhs = (h * (PF(gga, b, xu) + PF(a, ggb, xu))).sum()
    torch.testing.assert_close(lhs, rhs, rtol=rtol * 10, atol=atol * 10)
    # mix adjoints
    xy = mk(B, P, K, I)
    lhs = (ext.mix_dbl_bwd_grad_y(go, w, ggw, gates, ggg) * xy).sum()
    rhs = (go * (_ref_mix(xy, ggw, gates) + _ref_mix(xy, w, ggg))).sum()
    torch.testing.assert_close(lhs, rhs, rtol=rtol * 10, atol=atol * 10)
    xw = mk(P, O, I)
    lhs = (ext.mix_dbl_bwd_grad_w(go, y, ggy, gates, ggg) * xw).sum()
    rhs = (go * (_ref_mix(ggy, xw, gates) + _ref_mix(y, xw, ggg))).sum()
    torch.testing.assert_close(lhs, rhs, rtol=rtol * 10, atol=atol * 10)
    xg = mk(B, P)
    lhs = (ext.mix_dbl_bwd_grad_g(go, y, ggy, w, ggw) * xg).sum()
    rhs = (go * (_ref_mix(ggy, w, xg) + _ref_mix(y, ggw, xg))).sum()
    torch.testing.assert_close(lhs, rhs, rtol=rtol * 10, atol=atol * 10)


def test_cpu_tensors_are_rejected():
    a = torch.zeros(2, 2, 3)
    with pytest.raises(RuntimeError, match="CUDA"):
        ext.project_bucket_forward(a, torch.zeros(2, 1, 3), torch.zeros(9, 3), 1)
