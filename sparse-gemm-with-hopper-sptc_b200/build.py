"""Build recipes for the sp24 shared library (nvcc, sm_100a, in-tree output).

``python sparse-gemm-with-hopper-sptc_b200/build.py`` builds ``lib/libsp24.so``.
The library links the CUDA runtime statically and resolves the driver's
tensor-map encoder at run time, so it loads on a machine without a GPU.
"""
from __future__ import annotations

import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
CSRC = os.path.join(HERE, "csrc")
LIBDIR = os.path.join(HERE, "lib")
NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
COMMON = ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC", "-Xcompiler", "-Wall"]

LIB_SOURCES = ["sp24_api.cu"]
LIB_DEPS = ["sp24_api.cu", "sp24_gemm_kernel.cuh", "sp24_gemm2sm_kernel.cuh", "sp24_prep.cuh",
            "sp24_ptx.cuh"]


def _stale(target: str, deps) -> bool:
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(d) > t for d in deps)


def _run(cmd, cwd=None) -> None:
    print("+", " ".join(cmd), flush=True)
    subprocess.run(cmd, check=True, cwd=cwd)


def build_lib(force: bool = False) -> str:
    os.makedirs(LIBDIR, exist_ok=True)
    out = os.path.join(LIBDIR, "libsp24.so")
    deps = [os.path.join(CSRC, f) for f in LIB_DEPS] + [os.path.join(ROOT, "include", "sp24.h")]
    if force or _stale(out, deps):
        tmp = out + ".tmp"
        _run([NVCC, *ARCH, *COMMON, "-shared", "-o", tmp,
              *[os.path.join(CSRC, s) for s in LIB_SOURCES]])
        os.replace(tmp, out)
    return out


if __name__ == "__main__":
    build_lib(force="--force" in sys.argv)
