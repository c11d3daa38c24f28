"""ctypes binding of ``libfsctep_b200.so`` (the C ABI declared in ``include/fsctep_b200.h``).

The library is required: importing a compute entry point without it raises.  There is
no CPU fallback anywhere in the package.
"""

from __future__ import annotations

import ctypes as C
import os
import threading

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "_lib", "libfsctep_b200.so")

_lib = None
_lock = threading.Lock()

P = C.c_void_p
I64 = C.c_int64
I32 = C.c_int32

FSC_F32, FSC_F64 = 0, 1


class IctdConfig(C.Structure):
    _fields_ = [("channels", I32), ("lmax", I32), ("num_interaction", I32), ("number_of_basis", I32),
                ("basis_kind", I32), ("max_radius", C.c_float), ("num_species", I32), ("output_size", I32),
                ("invariant_channels", I32), ("n_hidden", I32), ("hidden", I32 * 4), ("n_out", I32), ("o3", I32)]


class IctdWeights(C.Structure):
    _fields_ = [("tables", P), ("ai", P), ("vsp", P), ("rad_w1", P), ("rad_b1", P), ("rad_w2", P),
                ("rad_b2", P), ("rad_w3", P), ("rad_b3", P), ("mix_fwd", P), ("mix_bwd", P), ("mix_dx", P),
                ("wread_p", P), ("wread_s", P), ("pairs", P), ("xmap", P), ("xinv", P), ("wimg_fwd", P), ("wimg_bwd", P), ("mn_in_g", P), ("mn_in_b", P),
                ("mn_w", P * 4), ("mn_b", P * 4), ("mn_g", P * 4), ("mn_beta", P * 4), ("out_v", P),
                ("out_c0", C.c_float)]


class SparseConfig(C.Structure):
    _fields_ = [("channels", I32), ("lmax", I32), ("num_interaction", I32), ("number_of_basis", I32),
                ("basis_kind", I32), ("max_radius", C.c_float), ("num_species", I32), ("invariant_channels", I32),
                ("n_hidden", I32), ("hidden", I32 * 4), ("n_out", I32), ("avg_num_neighbors", C.c_float)]


class SparseWeights(C.Structure):
    _fields_ = [("rad_w1", P), ("rad_b1", P), ("rad_w2", P), ("rad_b2", P), ("pair_k", P), ("mix", P),
                ("mixT", P), ("wread_p", P), ("wread_s", P), ("pairs", P), ("mn_in_g", P), ("mn_in_b", P),
                ("mn_w", P * 4), ("mn_b", P * 4), ("mn_g", P * 4), ("mn_beta", P * 4), ("out_v", P),
                ("out_c0", C.c_float)]


class Graph(C.Structure):
    _fields_ = [("num_atoms", I64), ("num_local", I64), ("num_edges", I64), ("num_graphs", I64), ("pos", P),
                ("species", P), ("batch", P), ("cell", P), ("row_ptr", P), ("src", P), ("shift", P),
                ("tr_ptr", P), ("tr_eid", P), ("energy_weight", P), ("field", P), ("layer_atoms", P)]


class IctdOutputs(C.Structure):
    _fields_ = [("energy", P), ("atom_energy", P), ("forces", P), ("virial", P), ("edge_grad", P),
                ("cell_grad", P)]


_PROTOS = {
    "fsc_last_error": (C.c_char_p, []),
    "fsc_version": (C.c_int, []),
    "fsc_has_cuda": (C.c_int, []),
    "fsc_project_bucket_forward": (C.c_int, [C.c_int, P, P, P, P] + [I64] * 7 + [P]),
    "fsc_project_bucket_transpose_a": (C.c_int, [C.c_int, P, P, P, P] + [I64] * 7 + [P]),
    "fsc_project_bucket_transpose_b": (C.c_int, [C.c_int, P, P, P, P] + [I64] * 7 + [P]),
    "fsc_project_bucket_transpose_u": (C.c_int, [C.c_int, P, P, P, P] + [I64] * 7 + [P]),
    "fsc_mix_bucket_forward": (C.c_int, [C.c_int, P, P, P, P] + [I64] * 5 + [P]),
    "fsc_mix_bucket_transpose_y": (C.c_int, [C.c_int, P, P, P, P] + [I64] * 5 + [P]),
    "fsc_mix_bucket_transpose_w": (C.c_int, [C.c_int, P, P, P, P] + [I64] * 5 + [P]),
    "fsc_mix_bucket_transpose_g": (C.c_int, [C.c_int, P, P, P, P] + [I64] * 5 + [P]),
    "fsc_bucketed_tp_forward": (C.c_int, [C.c_int, P, P, P, P, P, P] + [I64] * 8 + [P]),
    "fsc_project_dbl_bwd_grad_h": (C.c_int, [C.c_int] + [P] * 7 + [I64] * 7 + [P]),
    "fsc_project_dbl_bwd_grad_a": (C.c_int, [C.c_int] + [P] * 6 + [I64] * 7 + [P]),
    "fsc_project_dbl_bwd_grad_b": (C.c_int, [C.c_int] + [P] * 6 + [I64] * 7 + [P]),
    "fsc_project_dbl_bwd_grad_u": (C.c_int, [C.c_int] + [P] * 6 + [I64] * 7 + [P]),
    "fsc_mix_dbl_bwd_grad_g_out": (C.c_int, [C.c_int] + [P] * 7 + [I64] * 5 + [P]),
    "fsc_mix_dbl_bwd_grad_y": (C.c_int, [C.c_int] + [P] * 6 + [I64] * 5 + [P]),
    "fsc_mix_dbl_bwd_grad_w": (C.c_int, [C.c_int] + [P] * 6 + [I64] * 5 + [P]),
    "fsc_mix_dbl_bwd_grad_g": (C.c_int, [C.c_int] + [P] * 6 + [I64] * 5 + [P]),
    "fsc_neighbor_workspace_bytes": (C.c_size_t, [I64, I64]),
    "fsc_neighbor_count": (C.c_int, [P, P, P, I64, I64, P, C.c_double, P, P, P, C.c_size_t, P]),
    "fsc_neighbor_fill": (C.c_int, [P, P, P, I64, I64, P, C.c_double, P, P, P, I64, P, C.c_size_t, P]),
    "fsc_csr_transpose_workspace_bytes": (C.c_size_t, [I64, I64]),
    "fsc_csr_transpose": (C.c_int, [P, P, I64, I64, P, P, P, C.c_size_t, P]),
    "fsc_csr_transpose_static": (C.c_int, [P, P, I64, I64, P, P, P]),
    "fsc_neighbor_cap_workspace_bytes": (C.c_size_t, [I64, I64]),
    "fsc_neighbor_cap": (C.c_int, [P, P, P, I64, I64, P, P, C.c_int, P, P, P, P, P, C.c_size_t, P]),
    "fsc_ictd_tables_floats": (I64, []),
    "fsc_ictd_workspace_bytes": (C.c_size_t, [C.POINTER(IctdConfig), I64, I64]),
    "fsc_ictd_energy_forces": (C.c_int, [C.POINTER(IctdConfig), C.POINTER(IctdWeights), C.POINTER(Graph),
                                         C.POINTER(IctdOutputs), P, C.c_size_t, P]),
    "fsc_ictd_forward": (C.c_int, [C.POINTER(IctdConfig), C.POINTER(IctdWeights), C.POINTER(Graph), P, P, P,
                                   C.c_size_t, P]),
    "fsc_ictd_backward": (C.c_int, [C.POINTER(IctdConfig), C.POINTER(IctdWeights), C.POINTER(Graph),
                                    C.POINTER(IctdOutputs), P, C.c_size_t, P]),
    "fsc_ictd_status": (C.c_int, [C.POINTER(IctdConfig), I64, I64, P, P, C.POINTER(C.c_int)]),
    "fsc_ictd_forward_step": (C.c_int, [C.POINTER(IctdConfig), C.POINTER(IctdWeights), C.POINTER(Graph), C.c_int,
                                        P, P, P, C.c_size_t, P]),
    "fsc_ictd_backward_step": (C.c_int, [C.POINTER(IctdConfig), C.POINTER(IctdWeights), C.POINTER(Graph), C.c_int,
                                         C.POINTER(IctdOutputs), P, C.c_size_t, P]),
    "fsc_ictd_feature_buffer": (C.c_int, [C.POINTER(IctdConfig), I64, I64, P, C.c_int, C.c_int,
                                          C.POINTER(C.c_void_p)]),
    "fsc_ictd_set_readout_path": (None, [C.c_int]),
    "fsc_sparse_workspace_bytes": (C.c_size_t, [C.POINTER(SparseConfig), I64, I64]),
    "fsc_sparse_forward": (C.c_int, [C.POINTER(SparseConfig), C.POINTER(SparseWeights), C.POINTER(Graph), P, P, P,
                                     C.c_size_t, P]),
    "fsc_sparse_backward": (C.c_int, [C.POINTER(SparseConfig), C.POINTER(SparseWeights), C.POINTER(Graph),
                                      C.POINTER(IctdOutputs), P, C.c_size_t, P]),
    "fsc_sparse_status": (C.c_int, [C.POINTER(SparseConfig), I64, I64, P, P, C.POINTER(C.c_int)]),
    "fsc_sparse_forward_step": (C.c_int, [C.POINTER(SparseConfig), C.POINTER(SparseWeights), C.POINTER(Graph),
                                          C.c_int, P, P, P, C.c_size_t, P]),
    "fsc_sparse_backward_step": (C.c_int, [C.POINTER(SparseConfig), C.POINTER(SparseWeights), C.POINTER(Graph),
                                           C.c_int, C.POINTER(IctdOutputs), P, C.c_size_t, P]),
    "fsc_sparse_feature_buffer": (C.c_int, [C.POINTER(SparseConfig), I64, I64, P, C.c_int, C.c_int,
                                            C.POINTER(C.c_void_p)]),
    "fsc_ictd_heads": (C.c_int, [P, P, P, C.c_int, P, P, P, P, C.c_size_t, P]),
    "fsc_ictd_set_radial_path": (None, [C.c_int]),
    "fsc_ictd_set_gemm_path": (None, [C.c_int]),
    "fsc_ictd_set_conv2_path": (None, [C.c_int]),
    "fsc_fp32_fma_probe": (C.c_int, [C.c_int, C.c_int, C.c_int, P, C.POINTER(C.c_double), P]),
    "fsc_bounded_wait_probe": (C.c_int, [C.c_int, C.c_int, P, P]),
    "fsc_gemm_tc_plan": (C.c_int, [C.c_int, C.c_int, C.c_int, C.POINTER(C.c_int), C.POINTER(C.c_int)]),
    "fsc_profile_enable": (None, [C.c_int]),
    "fsc_profile_read": (C.c_int, [C.POINTER(C.c_char_p), C.POINTER(C.c_float), C.c_int]),
    "fsc_ictd_energy": (C.c_int, [C.POINTER(IctdConfig), C.POINTER(IctdWeights), C.POINTER(Graph), P, P, P,
                                  C.c_size_t, P]),
}


def exported_symbols():
    return sorted(_PROTOS)


def lib():
    """Load the library (once); raises if it is missing -- there is no fallback."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is None:
            if not os.path.exists(LIB_PATH):
                raise RuntimeError(f"fsctep_b200 native library not built: {LIB_PATH} "
                                   "(run `python -m fsctep_b200.build`)")
            handle = C.CDLL(LIB_PATH)
            for name, (res, args) in _PROTOS.items():
                fn = getattr(handle, name)
                fn.restype = res
                fn.argtypes = args
            _lib = handle
    return _lib


class NativeError(RuntimeError):
    pass


def check(status: int, what: str) -> None:
    if status != 0:
        msg = lib().fsc_last_error().decode(errors="replace")
        raise NativeError(f"{what} failed (status {status}): {msg}")


def stream_ptr(device=None):
    import torch

    return P(torch.cuda.current_stream(device).cuda_stream)


def profile_enable(on: bool) -> None:
    lib().fsc_profile_enable(1 if on else 0)


def profile_read(max_stages: int = 64):
    """[(stage name, ms)] recorded since the last enable/read (synchronises)."""
    names = (C.c_char_p * max_stages)()
    ms = (C.c_float * max_stages)()
    n = lib().fsc_profile_read(names, ms, max_stages)
    if n < 0:
        raise NativeError("fsc_profile_read failed")
    return [(names[i].decode(), float(ms[i])) for i in range(n)]


def ptr(t):
    return P(0) if t is None else P(t.data_ptr())
