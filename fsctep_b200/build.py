"""Build the sm_100a shared library ``fsctep_b200/_lib/libfsctep_b200.so`` with nvcc, and the
TorchScript op library ``fsctep_b200/_lib/libfsctep_b200_torch.so`` with g++.

The main library is plain CUDA C++ behind the C ABI in ``include/fsctep_b200.h`` (no torch
types); Python loads it with ctypes.  The op library registers ``fsctep::ictd_atom_energy``
(TORCH_LIBRARY) on top of it for core.pt; it links libtorch and the main library, not libpython.
Run ``python -m fsctep_b200.build`` (or ``__graft_entry__.build()``).  Objects are compiled in
parallel and linked once.
"""

from __future__ import annotations

import concurrent.futures as cf
import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
CSRC = os.path.join(HERE, "csrc")
LIBDIR = os.path.join(HERE, "_lib")
LIB = os.path.join(LIBDIR, "libfsctep_b200.so")
OBJDIR = os.path.join(ROOT, "_build", "obj")
OPSRC = os.path.join(HERE, "torch_ops", "ictd_op.cpp")
OPLIB = os.path.join(LIBDIR, "libfsctep_b200_torch.so")

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC", "--expt-relaxed-constexpr",
         "-I" + os.path.join(ROOT, "include"), "-I" + CSRC]


def nvcc() -> str:
    for cand in (shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found")


def sources():
    return sorted(os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith(".cu"))


def _compile(src: str, verbose: bool) -> str:
    obj = os.path.join(OBJDIR, os.path.basename(src) + ".o")
    cmd = [nvcc(), *ARCH, *FLAGS, "-c", src, "-o", obj]
    if verbose:
        cmd.insert(1, "-Xptxas=-v")
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"nvcc failed for {src}:\n{res.stdout}\n{res.stderr}")
    if verbose and res.stderr:
        sys.stderr.write(res.stderr)
    return obj


def build_torch_ops(force: bool = False) -> str:
    """g++ build of the TORCH_LIBRARY op library against the installed torch."""
    import torch
    from torch.utils import cpp_extension as ce

    deps = [OPSRC, LIB, os.path.join(ROOT, "include", "fsctep_b200.h")]
    if not force and os.path.exists(OPLIB) and all(os.path.getmtime(d) <= os.path.getmtime(OPLIB) for d in deps):
        return OPLIB
    torch_lib = os.path.join(os.path.dirname(torch.__file__), "lib")
    cuda_home = ce.CUDA_HOME or "/usr/local/cuda"
    incs = [os.path.join(os.path.dirname(torch.__file__), "include"),
            os.path.join(os.path.dirname(torch.__file__), "include", "torch", "csrc", "api", "include"),
            os.path.join(cuda_home, "include"), os.path.join(ROOT, "include")]
    abi = int(torch._C._GLIBCXX_USE_CXX11_ABI)
    tmp = OPLIB + ".tmp"
    cmd = ["g++", "-O2", "-std=c++17", "-fPIC", "-shared", f"-D_GLIBCXX_USE_CXX11_ABI={abi}",
           *[f"-I{i}" for i in incs], OPSRC, "-o", tmp,
           f"-L{torch_lib}", "-ltorch", "-ltorch_cpu", "-ltorch_cuda", "-lc10", "-lc10_cuda",
           f"-L{LIBDIR}", "-lfsctep_b200", f"-L{os.path.join(cuda_home, 'lib64')}", "-lcudart",
           "-Wl,-rpath,$ORIGIN", f"-Wl,-rpath,{torch_lib}"]
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"g++ failed for {OPSRC}:\n{res.stdout}\n{res.stderr}")
    os.replace(tmp, OPLIB)
    return OPLIB


def build(verbose: bool = False, force: bool = False, torch_ops: bool = True) -> str:
    lib = _build_main(verbose, force)
    if torch_ops:
        build_torch_ops(force)
    return lib


def _build_main(verbose: bool = False, force: bool = False) -> str:
    os.makedirs(OBJDIR, exist_ok=True)
    os.makedirs(LIBDIR, exist_ok=True)
    srcs = sources()
    deps = srcs + [os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith(".cuh")]
    deps.append(os.path.join(ROOT, "include", "fsctep_b200.h"))
    if not force and os.path.exists(LIB):
        lib_t = os.path.getmtime(LIB)
        if all(os.path.getmtime(d) <= lib_t for d in deps):
            return LIB
    with cf.ThreadPoolExecutor(max_workers=min(8, len(srcs))) as ex:
        objs = list(ex.map(lambda s: _compile(s, verbose), srcs))
    tmp = LIB + ".tmp"
    cmd = [nvcc(), *ARCH, "-shared", "-o", tmp, *objs, "-lcudart"]
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"link failed:\n{res.stdout}\n{res.stderr}")
    os.replace(tmp, LIB)
    return LIB


if __name__ == "__main__":
    print(build(verbose="-v" in sys.argv, force="-f" in sys.argv))
