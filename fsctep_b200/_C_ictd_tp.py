"""Drop-in for the reference extension module ``molecular_force_field._C_ictd_tp``.

Same operator names, argument meaning, output shapes and error behaviour as the pybind
module of the reference (``csrc/ictd_tp.cpp:137-523``): inputs are borrowed (made
contiguous when needed), outputs are freshly allocated on the input device, shape errors
raise ``RuntimeError``.  The kernels are the sm_100a CUDA implementations in
``libfsctep_b200.so`` called through the C ABI on the *current* CUDA stream (the
reference launched on the legacy default stream).  Differences by design: inputs must be
CUDA tensors (there is no CPU path; CPU tensors raise ``RuntimeError``), and any
``mul_in2`` is supported on the GPU (the reference CUDA path needs ``mul_in2 == 1``).
"""

from __future__ import annotations

import torch

from fsctep_b200 import _native as N

__all__ = [
    "project_bucket_forward", "project_bucket_transpose_a", "project_bucket_transpose_b",
    "project_bucket_transpose_u", "mix_bucket_forward", "mix_bucket_transpose_y", "mix_bucket_transpose_w",
    "mix_bucket_transpose_g", "bucketed_tp_forward", "project_dbl_bwd_grad_h", "project_dbl_bwd_grad_a",
    "project_dbl_bwd_grad_b", "project_dbl_bwd_grad_u", "mix_dbl_bwd_grad_g_out", "mix_dbl_bwd_grad_y",
    "mix_dbl_bwd_grad_w", "mix_dbl_bwd_grad_g", "has_cuda",
]


def has_cuda() -> bool:
    """True: this module's operators run the sm_100a CUDA kernels."""
    return bool(N.lib().fsc_has_cuda())


def _check(cond, msg):
    if not cond:
        raise RuntimeError(msg)


def _prep(*ts):
    ref = ts[0]
    _check(ref.is_cuda, "fsctep_b200 _C_ictd_tp operators require CUDA tensors")
    _check(ref.dtype in (torch.float32, torch.float64), "only float32/float64 are supported")
    out = []
    for t in ts:
        _check(t.device == ref.device, "all tensors must be on the same device")
        _check(t.dtype == ref.dtype, "all tensors must have the same dtype")
        out.append(t.contiguous())
    return out


def _dt(t):
    return N.FSC_F32 if t.dtype == torch.float32 else N.FSC_F64


def _st(t):
    return N.stream_ptr(t.device)


def _proj_dims(a, b, u, num_paths):
    _check(a.dim() == 3, "a must have shape (B, mul_in1, m1)")
    _check(b.dim() == 3, "b must have shape (B, mul_in2, m2)")
    _check(u.dim() == 2, "u_bucket must have shape (m1*m2, P*kdim)")
    _check(b.size(0) == a.size(0), "a and b batch dimensions must match")
    _check(u.size(0) == a.size(2) * b.size(2), "u_bucket first dim must equal m1*m2")
    _check(num_paths > 0, "num_paths must be positive")
    _check(u.size(1) % num_paths == 0, "u_bucket second dim must be divisible by num_paths")
    return a.size(0), a.size(1), b.size(1), a.size(2), b.size(2), int(num_paths), u.size(1) // num_paths


def project_bucket_forward(a, b, u_bucket, num_paths):
    a, b, u = _prep(a, b, u_bucket)
    B, I, J, m1, m2, P, K = _proj_dims(a, b, u, num_paths)
    y = torch.empty(B, P, K, I * J, device=a.device, dtype=a.dtype)
    N.check(N.lib().fsc_project_bucket_forward(_dt(a), N.ptr(a), N.ptr(b), N.ptr(u), N.ptr(y), B, I, J, m1, m2, P, K,
                                               _st(a)), "project_bucket_forward")
    return y


def _grad_y_dims(grad_y):
    _check(grad_y.dim() == 4, "grad_y must have shape (B, P, kdim, IJ)")
    return grad_y.size(0), grad_y.size(1), grad_y.size(2), grad_y.size(3)


def project_bucket_transpose_a(grad_y, b, u_bucket):
    grad_y, b, u = _prep(grad_y, b, u_bucket)
    _check(b.dim() == 3, "b must have shape (B, mul_in2, m2)")
    _check(u.dim() == 2, "u_bucket must have shape (m1*m2, P*kdim)")
    B, P, K, IJ = _grad_y_dims(grad_y)
    _check(B == b.size(0), "grad_y batch must match b")
    J, m2 = b.size(1), b.size(2)
    _check(IJ % J == 0, "grad_y IJ dim must be divisible by mul_in2")
    _check(u.size(0) % m2 == 0, "u_bucket first dim must factor into m1*m2")
    I, m1 = IJ // J, u.size(0) // m2
    _check(u.size(1) == P * K, "u_bucket second dim must equal P*kdim")
    out = torch.empty(B, I, m1, device=b.device, dtype=b.dtype)
    N.check(N.lib().fsc_project_bucket_transpose_a(_dt(b), N.ptr(grad_y), N.ptr(b), N.ptr(u), N.ptr(out), B, I, J, m1,
                                                   m2, P, K, _st(b)), "project_bucket_transpose_a")
    return out


def project_bucket_transpose_b(grad_y, a, u_bucket):
    grad_y, a, u = _prep(grad_y, a, u_bucket)
    _check(a.dim() == 3, "a must have shape (B, mul_in1, m1)")
    _check(u.dim() == 2, "u_bucket must have shape (m1*m2, P*kdim)")
    B, P, K, IJ = _grad_y_dims(grad_y)
    _check(B == a.size(0), "grad_y batch must match a")
    I, m1 = a.size(1), a.size(2)
    _check(IJ % I == 0, "grad_y IJ dim must be divisible by mul_in1")
    _check(u.size(0) % m1 == 0, "u_bucket first dim must factor into m1*m2")
    J, m2 = IJ // I, u.size(0) // m1
    _check(u.size(1) == P * K, "u_bucket second dim must equal P*kdim")
    out = torch.empty(B, J, m2, device=a.device, dtype=a.dtype)
    N.check(N.lib().fsc_project_bucket_transpose_b(_dt(a), N.ptr(grad_y), N.ptr(a), N.ptr(u), N.ptr(out), B, I, J, m1,
                                                   m2, P, K, _st(a)), "project_bucket_transpose_b")
    return out


def project_bucket_transpose_u(grad_y, a, b):
    grad_y, a, b = _prep(grad_y, a, b)
    _check(a.dim() == 3 and b.dim() == 3, "a/b must be 3-D")
    B, P, K, IJ = _grad_y_dims(grad_y)
    I, m1, J, m2 = a.size(1), a.size(2), b.size(1), b.size(2)
    _check(IJ == I * J, "grad_y last dim must equal mul_in1*mul_in2")
    out = torch.empty(m1 * m2, P * K, device=a.device, dtype=a.dtype)
    N.check(N.lib().fsc_project_bucket_transpose_u(_dt(a), N.ptr(grad_y), N.ptr(a), N.ptr(b), N.ptr(out), B, I, J, m1,
                                                   m2, P, K, _st(a)), "project_bucket_transpose_u")
    return out


def _mix_dims(y, w, gates):
    _check(y.dim() == 4, "y must have shape (B, P, kdim, IJ)")
    _check(w.dim() == 3, "w must have shape (P, mul_out, IJ)")
    _check(gates.dim() == 2, "gates must have shape (B, P)")
    _check(y.size(0) == gates.size(0), "gates batch dim must match y")
    _check(y.size(1) == w.size(0), "w path dim must match y")
    _check(y.size(1) == gates.size(1), "gates path dim must match y")
    _check(y.size(3) == w.size(2), "w IJ dim must match y")
    return y.size(0), y.size(1), y.size(2), y.size(3), w.size(1)


def mix_bucket_forward(y, w, gates):
    y, w, gates = _prep(y, w, gates)
    B, P, K, IJ, O = _mix_dims(y, w, gates)
    out = torch.empty(B, O, K, device=y.device, dtype=y.dtype)
    N.check(N.lib().fsc_mix_bucket_forward(_dt(y), N.ptr(y), N.ptr(w), N.ptr(gates), N.ptr(out), B, P, K, IJ, O,
                                           _st(y)), "mix_bucket_forward")
    return out


def mix_bucket_transpose_y(grad_out, w, gates):
    grad_out, w, gates = _prep(grad_out, w, gates)
    _check(grad_out.dim() == 3, "grad_out must have shape (B, O, kdim)")
    _check(w.dim() == 3, "w must have shape (P, O, IJ)")
    _check(gates.dim() == 2, "gates must have shape (B, P)")
    B, O, K = grad_out.shape
    P, IJ = w.size(0), w.size(2)
    _check(w.size(1) == O, "w output dim must match grad_out")
    _check(gates.size(0) == B and gates.size(1) == P, "gates must match grad_out and w")
    out = torch.empty(B, P, K, IJ, device=w.device, dtype=w.dtype)
    N.check(N.lib().fsc_mix_bucket_transpose_y(_dt(w), N.ptr(grad_out), N.ptr(w), N.ptr(gates), N.ptr(out), B, P, K,
                                               IJ, O, _st(w)), "mix_bucket_transpose_y")
    return out


def mix_bucket_transpose_w(grad_out, y, gates):
    grad_out, y, gates = _prep(grad_out, y, gates)
    _check(grad_out.dim() == 3 and y.dim() == 4 and gates.dim() == 2, "bad ranks")
    B, P, K, IJ = y.shape
    O = grad_out.size(1)
    _check(gates.shape == (B, P) and grad_out.size(0) == B and grad_out.size(2) == K, "shape mismatch")
    out = torch.empty(P, O, IJ, device=y.device, dtype=y.dtype)
    N.check(N.lib().fsc_mix_bucket_transpose_w(_dt(y), N.ptr(grad_out), N.ptr(y), N.ptr(gates), N.ptr(out), B, P, K,
                                               IJ, O, _st(y)), "mix_bucket_transpose_w")
    return out


def mix_bucket_transpose_g(grad_out, y, w):
    grad_out, y, w = _prep(grad_out, y, w)
    _check(grad_out.dim() == 3, "grad_out must have shape (B, O, kdim)")
    _check(y.dim() == 4, "y must have shape (B, P, kdim, IJ)")
    _check(w.dim() == 3, "w must have shape (P, O, IJ)")
    B, P, K, IJ = y.shape
    O = grad_out.size(1)
    _check(grad_out.size(0) == B and grad_out.size(2) == K, "grad_out must match y")
    _check(w.size(0) == P and w.size(1) == O and w.size(2) == IJ, "w must match y and grad_out")
    out = torch.empty(B, P, device=y.device, dtype=y.dtype)
    N.check(N.lib().fsc_mix_bucket_transpose_g(_dt(y), N.ptr(grad_out), N.ptr(y), N.ptr(w), N.ptr(out), B, P, K, IJ,
                                               O, _st(y)), "mix_bucket_transpose_g")
    return out


def bucketed_tp_forward(a, b, u_bucket, w, gates):
    a, b, u, w, gates = _prep(a, b, u_bucket, w, gates)
    _check(w.dim() == 3, "w must have shape (P, mul_out, IJ)")
    _check(gates.dim() == 2, "gates must have shape (B, P)")
    P = w.size(0)
    _check(gates.size(1) == P, "gates path dim must match w")
    B, I, J, m1, m2, P, K = _proj_dims(a, b, u, P)
    _check(w.size(2) == I * J, "w IJ dim must match")
    O = w.size(1)
    out = torch.empty(B, O, K, device=a.device, dtype=a.dtype)
    N.check(N.lib().fsc_bucketed_tp_forward(_dt(a), N.ptr(a), N.ptr(b), N.ptr(u), N.ptr(w), N.ptr(gates), N.ptr(out),
                                            B, I, J, m1, m2, P, K, O, _st(a)), "bucketed_tp_forward")
    return out


def project_dbl_bwd_grad_h(a, gga, b, ggb, u, ggu, num_paths):
    a, gga, b, ggb, u, ggu = _prep(a, gga, b, ggb, u, ggu)
    B, I, J, m1, m2, P, K = _proj_dims(a, b, u, num_paths)
    out = torch.empty(B, P, K, I * J, device=a.device, dtype=a.dtype)
    N.check(N.lib().fsc_project_dbl_bwd_grad_h(_dt(a), N.ptr(a), N.ptr(gga), N.ptr(b), N.ptr(ggb), N.ptr(u),
                                               N.ptr(ggu), N.ptr(out), B, I, J, m1, m2, P, K, _st(a)),
            "project_dbl_bwd_grad_h")
    return out


def project_dbl_bwd_grad_a(h, b, ggb, u, ggu):
    h, b, ggb, u, ggu = _prep(h, b, ggb, u, ggu)
    B, P, K, IJ = _grad_y_dims(h)
    J, m2 = b.size(1), b.size(2)
    I, m1 = IJ // J, u.size(0) // m2
    out = torch.empty(B, I, m1, device=h.device, dtype=h.dtype)
    N.check(N.lib().fsc_project_dbl_bwd_grad_a(_dt(h), N.ptr(h), N.ptr(b), N.ptr(ggb), N.ptr(u), N.ptr(ggu),
                                               N.ptr(out), B, I, J, m1, m2, P, K, _st(h)), "project_dbl_bwd_grad_a")
    return out


def project_dbl_bwd_grad_b(h, a, gga, u, ggu):
    h, a, gga, u, ggu = _prep(h, a, gga, u, ggu)
    B, P, K, IJ = _grad_y_dims(h)
    I, m1 = a.size(1), a.size(2)
    J, m2 = IJ // I, u.size(0) // m1
    out = torch.empty(B, J, m2, device=h.device, dtype=h.dtype)
    N.check(N.lib().fsc_project_dbl_bwd_grad_b(_dt(h), N.ptr(h), N.ptr(a), N.ptr(gga), N.ptr(u), N.ptr(ggu),
                                               N.ptr(out), B, I, J, m1, m2, P, K, _st(h)), "project_dbl_bwd_grad_b")
    return out


def project_dbl_bwd_grad_u(h, a, gga, b, ggb):
    h, a, gga, b, ggb = _prep(h, a, gga, b, ggb)
    B, P, K, IJ = _grad_y_dims(h)
    I, m1, J, m2 = a.size(1), a.size(2), b.size(1), b.size(2)
    out = torch.empty(m1 * m2, P * K, device=h.device, dtype=h.dtype)
    N.check(N.lib().fsc_project_dbl_bwd_grad_u(_dt(h), N.ptr(h), N.ptr(a), N.ptr(gga), N.ptr(b), N.ptr(ggb),
                                               N.ptr(out), B, I, J, m1, m2, P, K, _st(h)), "project_dbl_bwd_grad_u")
    return out


def mix_dbl_bwd_grad_g_out(y, ggy, w, ggw, gates, ggg):
    y, ggy, w, ggw, gates, ggg = _prep(y, ggy, w, ggw, gates, ggg)
    B, P, K, IJ, O = _mix_dims(y, w, gates)
    out = torch.empty(B, O, K, device=y.device, dtype=y.dtype)
    N.check(N.lib().fsc_mix_dbl_bwd_grad_g_out(_dt(y), N.ptr(y), N.ptr(ggy), N.ptr(w), N.ptr(ggw), N.ptr(gates),
                                               N.ptr(ggg), N.ptr(out), B, P, K, IJ, O, _st(y)),
            "mix_dbl_bwd_grad_g_out")
    return out


def mix_dbl_bwd_grad_y(g_out, w, ggw, gates, ggg):
    g_out, w, ggw, gates, ggg = _prep(g_out, w, ggw, gates, ggg)
    B, O, K = g_out.shape
    P, IJ = w.size(0), w.size(2)
    out = torch.empty(B, P, K, IJ, device=w.device, dtype=w.dtype)
    N.check(N.lib().fsc_mix_dbl_bwd_grad_y(_dt(w), N.ptr(g_out), N.ptr(w), N.ptr(ggw), N.ptr(gates), N.ptr(ggg),
                                           N.ptr(out), B, P, K, IJ, O, _st(w)), "mix_dbl_bwd_grad_y")
    return out


def mix_dbl_bwd_grad_w(g_out, y, ggy, gates, ggg):
    g_out, y, ggy, gates, ggg = _prep(g_out, y, ggy, gates, ggg)
    B, P, K, IJ = y.shape
    O = g_out.size(1)
    out = torch.empty(P, O, IJ, device=y.device, dtype=y.dtype)
    N.check(N.lib().fsc_mix_dbl_bwd_grad_w(_dt(y), N.ptr(g_out), N.ptr(y), N.ptr(ggy), N.ptr(gates), N.ptr(ggg),
                                           N.ptr(out), B, P, K, IJ, O, _st(y)), "mix_dbl_bwd_grad_w")
    return out


def mix_dbl_bwd_grad_g(g_out, y, ggy, w, ggw):
    g_out, y, ggy, w, ggw = _prep(g_out, y, ggy, w, ggw)
    B, P, K, IJ = y.shape
    O = g_out.size(1)
    out = torch.empty(B, P, device=y.device, dtype=y.dtype)
    N.check(N.lib().fsc_mix_dbl_bwd_grad_g(_dt(y), N.ptr(g_out), N.ptr(y), N.ptr(ggy), N.ptr(w), N.ptr(ggw),
                                           N.ptr(out), B, P, K, IJ, O, _st(y)), "mix_dbl_bwd_grad_g")
    return out
