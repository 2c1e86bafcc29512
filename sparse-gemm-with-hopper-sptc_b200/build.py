"""Build recipes (nvcc, sm_100a, in-tree outputs).

  build_lib()      lib/libsp24.so — the product: kernels + C ABI.  The CUDA
                   runtime is linked statically and the driver's tensor-map
                   encoder is resolved at run time, so the library loads on a
                   machine without a GPU.
  build_dropin()   bin/<entry> — the reference's own per-dtype entry points
                   (mma_sp_wgmma_*.cu, compiled where they lie) against the
                   drop-in headers in dropin/, linked with -lsp24.  A quoted
                   include searches the including file's directory first, so
                   each main is reached through a symlink in _build/dropin/
                   that sits next to the drop-in headers.
  build_probe()    lib/libsp24_peak.so — the tensor-core rate probe that bench.py
                   and the tests use to measure the roofline's peak (measurement
                   infrastructure, not part of the C ABI).
  build_feed_probe() bin/sp24_feed_probe — the shared-memory feed probe: TMA
                   ring fill rates with a slot-holding consumer, from L2 and
                   from HBM (measurement only; run by hand).
  build_oracle()   oracle/lib + oracle/_ref (test infrastructure, see oracle/).

``python sparse-gemm-with-hopper-sptc_b200/build.py [--force]`` builds all.
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
LIB_DEPS = ["sp24_api.cu", "sp24_gemm_kernel.cuh", "sp24_gemm2sm_kernel.cuh",
            "sp24_gemm_splitk_kernel.cuh", "sp24_prep.cuh",
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


def build_probe(force: bool = False) -> str:
    os.makedirs(LIBDIR, exist_ok=True)
    out = os.path.join(LIBDIR, "libsp24_peak.so")
    deps = [os.path.join(CSRC, f) for f in LIB_DEPS + ["sp24_peak.cu"]]
    if force or _stale(out, deps):
        tmp = out + ".tmp"
        _run([NVCC, *ARCH, *COMMON, "-shared", "-o", tmp, os.path.join(CSRC, "sp24_peak.cu")])
        os.replace(tmp, out)
    return out


DROPIN = os.path.join(HERE, "dropin")
BINDIR = os.path.join(HERE, "bin")


def build_feed_probe(force: bool = False) -> str:
    os.makedirs(BINDIR, exist_ok=True)
    out = os.path.join(BINDIR, "sp24_feed_probe")
    src = os.path.join(CSRC, "sp24_feed_probe.cu")
    if force or _stale(out, [src, os.path.join(CSRC, "sp24_ptx.cuh")]):
        _run([NVCC, *ARCH, "-O3", "-std=c++17", "-lineinfo", src, "-o", out])
    return out
# The reference checkout: SP24_REF_DIR, else a `reference` directory beside
# the repository.  Only the drop-in and oracle builds read it, and only when
# it exists.
REF_DIR = os.environ.get("SP24_REF_DIR", os.path.join(os.path.dirname(ROOT), "reference"))


def dropin_mains(ref_dir: str = REF_DIR):
    """Reference entry points that include one of the two harness headers."""
    import glob
    out = []
    for path in sorted(glob.glob(os.path.join(ref_dir, "mma_sp_wgmma_*.cu"))):
        src = open(path).read()
        if '#include "wgmma_sp_raw_common.hpp"' in src or '#include "wgmma_sp_demo_common.hpp"' in src:
            out.append(path)
    return out


def build_dropin(ref_dir: str = REF_DIR, force: bool = False):
    """Compile every reference entry point against the drop-in headers."""
    mains = dropin_mains(ref_dir)
    if not mains:
        return []
    lib = build_lib()
    stage = os.path.join(HERE, "_build", "dropin")
    os.makedirs(stage, exist_ok=True)
    os.makedirs(BINDIR, exist_ok=True)
    for h in ("wgmma_sp_raw_common.hpp", "wgmma_sp_demo_common.hpp", "sp24_host_utils.hpp",
              "sp24_raw_kernel.cuh"):
        link = os.path.join(stage, h)
        if not os.path.islink(link):
            os.symlink(os.path.join(DROPIN, h), link)
    # sp24_raw_kernel.cuh includes ../csrc/sp24_ptx.cuh relative to the stage
    csrc_link = os.path.join(HERE, "_build", "csrc")
    if not os.path.islink(csrc_link):
        os.symlink(CSRC, csrc_link)
    deps = [lib, os.path.join(ROOT, "include", "sp24.h"), os.path.join(CSRC, "sp24_ptx.cuh")] + [
        os.path.join(DROPIN, h) for h in os.listdir(DROPIN)]
    built = []
    for path in mains:
        name = os.path.basename(path)[:-3]
        link = os.path.join(stage, name + ".cu")
        if os.path.islink(link) and os.readlink(link) != path:
            os.remove(link)
        if not os.path.islink(link):
            os.symlink(path, link)
        out = os.path.join(BINDIR, name)
        if force or _stale(out, deps + [path]):
            _run([NVCC, *ARCH, "-O2", "-std=c++17", "-I" + os.path.join(ROOT, "include"), link,
                  "-L" + LIBDIR, "-lsp24", "-Xlinker", "-rpath,$ORIGIN/../lib", "-o", out])
        built.append(out)
    return built


def build_raw_kernel_check(force: bool = False):
    """bin/raw_kernel_check (M = 64 form, the default) and
    bin/raw_kernel_check_m128 (M = 128 form): tests/raw_kernel_check.cu, the
    launchable wgmma_sp_raw_kernel run over the reference entry points'
    cases.  Test infrastructure."""
    lib = build_lib()
    os.makedirs(BINDIR, exist_ok=True)
    src = os.path.join(ROOT, "tests", "raw_kernel_check.cu")
    deps = [lib, src, os.path.join(CSRC, "sp24_ptx.cuh"), os.path.join(ROOT, "include", "sp24.h")] + [
        os.path.join(DROPIN, h) for h in os.listdir(DROPIN)]
    outs = []
    for name, layout in (("raw_kernel_check", 1), ("raw_kernel_check_m128", 0)):
        out = os.path.join(BINDIR, name)
        if force or _stale(out, deps):
            _run([NVCC, *ARCH, "-O2", "-std=c++17", f"-DSP24_RAW_LAYOUT={layout}",
                  "-I" + os.path.join(ROOT, "include"), "-I" + DROPIN, src,
                  "-L" + LIBDIR, "-lsp24", "-Xlinker", "-rpath,$ORIGIN/../lib", "-o", out])
        outs.append(out)
    return outs


def build_oracle(ref_dir: str = REF_DIR) -> None:
    """CPU oracle (always) and the reference harness (when the checkout exists)."""
    oracle_dir = os.path.join(ROOT, "oracle")
    targets = ["oracle"]
    if os.path.exists(os.path.join(ref_dir, "wgmma_sp_raw_common.hpp")):
        targets.append("ref")
    _run(["make", "-s", "-C", oracle_dir, *targets, "REF_DIR=" + ref_dir])


def build_all(force: bool = False) -> None:
    build_lib(force=force)
    build_probe(force=force)
    build_feed_probe(force=force)
    build_oracle()
    build_dropin(force=force)
    build_raw_kernel_check(force=force)


if __name__ == "__main__":
    build_all(force="--force" in sys.argv)
