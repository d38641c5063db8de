"""Build recipe for the native parts of periodicdent42_b200.

Produces, in-tree (next to this file):
  * ``libbsk_sm100.so`` -- the C-ABI library (include/bsk_capi.h): every sm_100a kernel plus its host
    launcher, compiled by nvcc with ``-gencode arch=compute_100a,code=sm_100a``; CUDA runtime linked
    statically so the library loads without a GPU.
  * ``_C.so`` -- the torch C++ extension ``periodicdent42_b200._C`` (the reference's
    ``blackwellsparsek._C`` surface, BlackwellSparseK/python/bsk_bindings.cpp:141-158), a thin layer that
    validates torch tensors and calls the C ABI.

Usage: ``python -m periodicdent42_b200.build [--capi-only]``.
"""
from __future__ import annotations

import os
import subprocess
import sys
import sysconfig

PKG_DIR = os.path.dirname(os.path.abspath(__file__))
REPO_DIR = os.path.dirname(PKG_DIR)
CSRC = os.path.join(PKG_DIR, "csrc")
INCLUDE = os.path.join(REPO_DIR, "include")
CAPI_LIB = os.path.join(PKG_DIR, "libbsk_sm100.so")
TORCH_EXT = os.path.join(PKG_DIR, "_C.so")

NVCC_ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
CAPI_SOURCES = [os.path.join(CSRC, "capi.cu")]
CAPI_DEPS = CAPI_SOURCES + sorted(
    os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith(".cuh")
) + [os.path.join(INCLUDE, "bsk_capi.h")]


def _nvcc() -> str:
    cuda_home = os.environ.get("CUDA_HOME", "/usr/local/cuda")
    return os.path.join(cuda_home, "bin", "nvcc")


def _stale(target: str, deps: list[str]) -> bool:
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(d) > t for d in deps if os.path.exists(d))


def _run(cmd: list[str]) -> None:
    r = subprocess.run(cmd, stdout=subprocess.PIPE, stderr=subprocess.STDOUT, text=True)
    if r.returncode != 0:
        sys.stderr.write(r.stdout)
        raise RuntimeError(f"build step failed ({r.returncode}): {' '.join(cmd[:3])} ...")


def build_capi(force: bool = False, extra: list[str] | None = None) -> str:
    """Compile the C-ABI library for sm_100a."""
    if not force and not _stale(CAPI_LIB, CAPI_DEPS):
        return CAPI_LIB
    tmp = CAPI_LIB + ".tmp"
    cmd = [_nvcc(), *NVCC_ARCH, "-lineinfo", "-O3", "-std=c++17", "-I", INCLUDE, "-shared", "-Xcompiler", "-fPIC",
           "-Xcompiler", "-fvisibility=default", *(extra or []), "-o", tmp, *CAPI_SOURCES]
    _run(cmd)
    os.replace(tmp, CAPI_LIB)
    return CAPI_LIB


def build_torch_ext(force: bool = False) -> str:
    """Compile the torch extension ``_C`` against torch's headers; links libbsk_sm100.so via $ORIGIN."""
    src = os.path.join(CSRC, "bindings.cpp")
    deps = [src, os.path.join(INCLUDE, "bsk_capi.h"), CAPI_LIB]
    if not force and not _stale(TORCH_EXT, deps):
        return TORCH_EXT
    import torch
    from torch.utils import cpp_extension

    inc = cpp_extension.include_paths()
    libdirs = cpp_extension.library_paths()
    abi = int(torch._C._GLIBCXX_USE_CXX11_ABI)
    py_inc = sysconfig.get_paths()["include"]
    cuda_inc = os.path.join(os.environ.get("CUDA_HOME", "/usr/local/cuda"), "include")
    tmp = TORCH_EXT + ".tmp"
    cmd = ["g++", "-O2", "-std=c++17", "-shared", "-fPIC", f"-D_GLIBCXX_USE_CXX11_ABI={abi}",
           "-DTORCH_EXTENSION_NAME=_C", "-DTORCH_API_INCLUDE_EXTENSION_H", "-w"]
    for d in inc + [py_inc, cuda_inc, INCLUDE]:
        cmd += ["-I", d]
    cmd += [src, "-o", tmp]
    for d in libdirs:
        cmd += ["-L", d]
    cmd += ["-L", PKG_DIR, "-lbsk_sm100", "-Wl,-rpath,$ORIGIN", "-lc10", "-ltorch", "-ltorch_cpu",
            "-ltorch_python", "-lc10_cuda", "-ltorch_cuda"]
    _run(cmd)
    os.replace(tmp, TORCH_EXT)
    return TORCH_EXT


def build_all(force: bool = False) -> None:
    build_capi(force=force)
    build_torch_ext(force=force)


if __name__ == "__main__":
    build_capi(force="--force" in sys.argv)
    if "--capi-only" not in sys.argv:
        build_torch_ext(force="--force" in sys.argv)
    print("built:", CAPI_LIB, "" if "--capi-only" in sys.argv else TORCH_EXT)
