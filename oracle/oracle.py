"""TEST INFRASTRUCTURE ONLY — Python face of the CPU oracle.

Loads ``oracle/lib/libsp24_oracle.so`` (our C++ restatement of the
reference's host algorithms, see sp24_oracle.cpp) and, when it was built,
``oracle/_ref/libsp24ref.so`` (the reference's own host code compiled where
it lies).  Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline
legs use this module; the product library never does.

Arrays cross as numpy raw bits: uint16 for fp16/bf16, uint8 for e4m3/e5m2.
Functions of one matrix take its element code (F16, BF16, E4M3, E5M2); the
library's mixed fp8 dtypes map to an (A, B) pair of them through ``elems``.
"""
from __future__ import annotations

import ctypes
import os
import re
from ctypes import c_float, c_int, c_longlong, c_size_t, c_uint, c_void_p

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ORACLE_LIB = os.path.join(HERE, "lib", "libsp24_oracle.so")
REF_LIB = os.path.join(HERE, "_ref", "libsp24ref.so")
REF_FP8_LIB = os.path.join(HERE, "_ref", "libsp24ref_fp8.so")

F16, BF16, E4M3, E5M2 = 0, 1, 2, 3
BITS = {F16: np.uint16, BF16: np.uint16, E4M3: np.uint8, E5M2: np.uint8}
NAMES = {"half": F16, "half_t": F16, "__nv_bfloat16": BF16, "bfloat16_t": BF16,
         "__nv_fp8_e4m3": E4M3, "__nv_fp8_e5m2": E5M2}

# Library dtype codes (include/sp24.h) -> (A element, B element).
LIB_E5M2_E4M3, LIB_E4M3_E5M2, LIB_E5M2 = 3, 4, 5
_ELEMS = {0: (F16, F16), 1: (BF16, BF16), 2: (E4M3, E4M3), LIB_E5M2_E4M3: (E5M2, E4M3),
          LIB_E4M3_E5M2: (E4M3, E5M2), LIB_E5M2: (E5M2, E5M2)}


def elems(lib_dtype: int):
    """(A element code, B element code) of a library dtype."""
    return _ELEMS[lib_dtype]

_o = None
_r = None


def _p(a):
    return a.ctypes.data_as(c_void_p)


def lib():
    global _o
    if _o is None:
        if not os.path.exists(ORACLE_LIB):
            raise FileNotFoundError(f"{ORACLE_LIB} missing: run `make -C oracle`")
        o = ctypes.CDLL(ORACLE_LIB)
        o.oracle_gen_new.restype = c_void_p
        o.oracle_gen_new.argtypes = [c_uint]
        o.oracle_gen_free.argtypes = [c_void_p]
        o.oracle_gen_structured_sparse_a.argtypes = [c_void_p, c_int, c_int, c_int, c_void_p]
        o.oracle_gen_pattern_sparse_a.argtypes = [c_int, c_int, c_int, c_void_p]
        o.oracle_gen_random_b.argtypes = [c_void_p, c_int, c_int, c_int, c_void_p]
        o.oracle_gen_pattern_b.argtypes = [c_int, c_int, c_int, c_void_p]
        o.oracle_compress.restype = c_longlong
        o.oracle_compress.argtypes = [c_int, c_void_p, c_int, c_int, c_void_p, c_void_p]
        o.oracle_decompress.argtypes = [c_int, c_void_p, c_void_p, c_int, c_int, c_void_p]
        o.oracle_gemm.argtypes = [c_int, c_void_p, c_void_p, c_void_p, c_int, c_int, c_int, c_int]
        o.oracle_gemm_mixed.argtypes = [c_int, c_int, c_void_p, c_void_p, c_void_p, c_int, c_int,
                                        c_int, c_int]
        o.oracle_gemm_rows.argtypes = [c_int, c_void_p, c_void_p, c_void_p, c_int, c_int, c_int,
                                       c_int, c_int]
        o.oracle_count_abs_errors.restype = c_int
        o.oracle_count_abs_errors.argtypes = [c_void_p, c_void_p, c_size_t, c_float]
        o.oracle_prune_2of4.argtypes = [c_int, c_void_p, c_int, c_int, c_void_p]
        o.oracle_meta_tc_image.argtypes = [c_int, c_void_p, c_int, c_int, c_void_p]
        o.oracle_quantize_e4m3.restype = c_float
        o.oracle_quantize_e4m3.argtypes = [c_void_p, c_size_t, c_void_p]
        o.oracle_quantize_e5m2.restype = c_float
        o.oracle_quantize_e5m2.argtypes = [c_void_p, c_size_t, c_void_p]
        o.oracle_to_float.argtypes = [c_int, c_void_p, c_size_t, c_void_p]
        o.oracle_gen_legacy.argtypes = [c_int, c_int, c_int, c_int, c_int, c_void_p, c_void_p]
        o.oracle_meta_k16_from_ref.argtypes = [c_void_p, c_int, c_int, c_void_p]
        o.oracle_from_float.argtypes = [c_int, c_void_p, c_size_t, c_void_p]
        _o = o
    return _o


def ref_available() -> bool:
    return os.path.exists(REF_LIB)


def ref_lib():
    global _r
    if _r is None:
        if not ref_available():
            raise FileNotFoundError(f"{REF_LIB} missing: run `make -C oracle ref`")
        r = ctypes.CDLL(REF_LIB)
        r.ref_gen_new.restype = c_void_p
        r.ref_gen_new.argtypes = [c_uint]
        r.ref_gen_free.argtypes = [c_void_p]
        r.ref_host_case.argtypes = [c_void_p, c_int, c_int, c_int, c_int, c_int, c_void_p,
                                    c_void_p, c_void_p, c_void_p, c_void_p]
        r.ref_compress.argtypes = [c_int, c_void_p, c_int, c_int, c_void_p, c_void_p]
        r.ref_cpu_gemm.argtypes = [c_int, c_void_p, c_void_p, c_void_p, c_int, c_int, c_int, c_int]
        _r = r
    return _r


REF_LEGACY_LIB = os.path.join(HERE, "_ref", "libsp24ref_legacy.so")
# The reference's legacy warp-level entry points, as ref_legacy_case numbers them.
LEGACY_FILES = ["mma_sp_m16n8k16_fp32fp16.cu", "mma_sp_m16n8k16_fp32bf16.cu",
                "mma_sp_m16n8k32_fp32fp16.cu", "mma_sp_m16n8k32_fp32bf16.cu"]


def legacy_dtype(which: int) -> int:
    return F16 if which in (0, 2) else BF16


def gen_legacy(which: int, m: int, n: int, k: int):
    """(A dense, B) of the legacy main `which` (mt19937(42), that main's order)."""
    dt = legacy_dtype(which)
    a = np.empty((m, k), np.uint16)
    b = np.empty((k, n), np.uint16)
    lib().oracle_gen_legacy(0 if which < 2 else 1, dt, m, n, k, _p(a), _p(b))
    return a, b


def meta_k16_from_ref(meta, m: int, k: int):
    """Reference-layout metadata bytes -> m16n8k16 words [k/16][m/2] (uint32)."""
    out = np.empty((k // 16, m // 2), np.uint32)
    lib().oracle_meta_k16_from_ref(_p(np.ascontiguousarray(meta)), m, k, _p(out))
    return out


def ref_legacy_available() -> bool:
    return os.path.exists(REF_LEGACY_LIB)


_rl = None


def _ref_legacy_lib():
    global _rl
    if _rl is None:
        r = ctypes.CDLL(REF_LEGACY_LIB)
        r.ref_legacy_case.restype = c_int
        r.ref_legacy_case.argtypes = [c_int, c_int, c_int, c_int] + [c_void_p] * 5
        r.ref_legacy_launch.restype = c_int
        r.ref_legacy_launch.argtypes = [c_int] + [c_void_p] * 4 + [c_int] * 3 + [c_void_p]
        _rl = r
    return _rl


def ref_legacy_launch(which: int, a_c: int, b: int, c: int, e: int, m: int, n: int, k: int,
                      stream: int = 0) -> int:
    """Launches the reference's own kernel of legacy main `which` (its
    mma.sp.sync kernel, built for sm_100a) on device pointers in that main's
    formats; returns the launch's CUDA error code (0 = launched)."""
    return _ref_legacy_lib().ref_legacy_launch(which, a_c, b, c, e, m, n, k, stream)


def ref_legacy_case(which: int, m: int, n: int, k: int, with_c: bool = True):
    """A legacy main replayed by the reference's own host code at m x n x k:
    (a, b, a_c, meta words, c or None); meta is [k/16][m/2] words for the
    m16n8k16 mains and [m][k/32] for the m16n8k32 ones."""
    r = _ref_legacy_lib()
    a = np.empty((m, k), np.uint16)
    b = np.empty((k, n), np.uint16)
    ac = np.empty((m, k // 2), np.uint16)
    e = np.empty((k // 16, m // 2) if which < 2 else (m, k // 32), np.uint32)
    c = np.empty((m, n), np.float32) if with_c else None
    rc = r.ref_legacy_case(which, m, n, k, _p(a), _p(b), _p(ac), _p(e),
                           _p(c) if with_c else None)
    assert rc == 0
    return a, b, ac, e, c


def ref_fp8_available() -> bool:
    return os.path.exists(REF_FP8_LIB)


def ref_fp8_suite():
    """Every case of the reference's mixed fp8 entry point
    (mma_sp_m16n8k64_fp32fp8.cu, run_one), produced by its own host code:
    dict of per-case arrays a (16x64 e5m2), b (64x8 e4m3, row-major K x N),
    a_c (16x32), meta (16x8 reference bytes), c (16x8 fp32), plus tags."""
    r = ctypes.CDLL(REF_FP8_LIB)
    r.ref_fp8_suite_size.restype = c_int
    r.ref_fp8_suite.restype = c_int
    r.ref_fp8_suite.argtypes = [c_void_p] * 5 + [ctypes.c_char_p, c_int]
    n = r.ref_fp8_suite_size()
    a = np.empty((n, 16, 64), np.uint8)
    bt = np.empty((n, 8, 64), np.uint8)
    ac = np.empty((n, 16, 32), np.uint8)
    e = np.empty((n, 16, 2), np.uint32)
    c = np.empty((n, 16, 8), np.float32)
    tags = ctypes.create_string_buffer(n * 64)
    got = r.ref_fp8_suite(_p(a), _p(bt), _p(ac), _p(e), _p(c), tags, 64)
    assert got == n
    names = [tags.raw[i * 64:(i + 1) * 64].split(b"\0")[0].decode() for i in range(n)]
    return {"a": a, "b": np.ascontiguousarray(bt.transpose(0, 2, 1)), "a_c": ac,
            "meta": e.view(np.uint8).reshape(n, 16, 8), "c": c, "tags": names}


# ------------------------------------------------------------------ generators
class Gen:
    """mt19937 stream shared by the cases of one suite (reference seed 1234)."""

    def __init__(self, seed: int = 1234):
        self.h = lib().oracle_gen_new(seed)

    def __del__(self):
        if getattr(self, "h", None):
            lib().oracle_gen_free(self.h)
            self.h = None


def host_case(gen: Gen, dt: int, m: int, n: int, k: int, use_pattern: bool):
    """One case of the reference suite runner: (a_dense, b, a_c, meta, c_ref)."""
    o = lib()
    a = np.empty(m * k, BITS[dt])
    b = np.empty(k * n, BITS[dt])
    if use_pattern:
        o.oracle_gen_pattern_sparse_a(dt, m, k, _p(a))
        o.oracle_gen_pattern_b(dt, k, n, _p(b))
    else:
        o.oracle_gen_structured_sparse_a(gen.h, dt, m, k, _p(a))
        o.oracle_gen_random_b(gen.h, dt, k, n, _p(b))
    a_c, meta = compress(dt, a.reshape(m, k))
    c = gemm(dt, a.reshape(m, k), b.reshape(k, n))
    return a.reshape(m, k), b.reshape(k, n), a_c, meta, c


def ref_host_case(rgen, dt: int, m: int, n: int, k: int, use_pattern: bool):
    """Same as host_case, computed by the reference's own host code."""
    r = ref_lib()
    a = np.empty(m * k, BITS[dt])
    b = np.empty(k * n, BITS[dt])
    ac = np.empty(m * k // 2, BITS[dt])
    e = np.empty(m * k // 8, np.uint8)
    c = np.empty(m * n, np.float32)
    r.ref_host_case(rgen, dt, m, n, k, 1 if use_pattern else 0, _p(a), _p(b), _p(ac), _p(e), _p(c))
    return a.reshape(m, k), b.reshape(k, n), ac.reshape(m, k // 2), e.reshape(m, k // 8), c.reshape(m, n)


# ------------------------------------------------------------------ algorithms
def compress(dt: int, a):
    a = np.ascontiguousarray(a)
    m, k = a.shape
    ac = np.empty((m, k // 2), BITS[dt])
    meta = np.empty((m, k // 8), np.uint8)
    bad = lib().oracle_compress(dt, _p(a), m, k, _p(ac), _p(meta))
    if bad >= 0:
        raise ValueError(f"not 2:4 at group {bad} (row {bad // (k // 4)}, group {bad % (k // 4)})")
    return ac, meta


def decompress(dt: int, a_c, meta, m: int, k: int):
    out = np.empty((m, k), BITS[dt])
    lib().oracle_decompress(dt, _p(np.ascontiguousarray(a_c)), _p(np.ascontiguousarray(meta)), m, k,
                            _p(out))
    return out


def gemm(dt: int, a, b, threads: int = 1):
    """fp32 sequential-k GEMM on the dense A (reference cpu_gemm_ref semantics)."""
    a = np.ascontiguousarray(a)
    b = np.ascontiguousarray(b)
    m, k = a.shape
    n = b.shape[1]
    c = np.empty((m, n), np.float32)
    lib().oracle_gemm(dt, _p(a), _p(b), _p(c), m, n, k, threads)
    return c


def gemm_mixed(dta: int, dtb: int, a, b, threads: int = 1):
    """As gemm, with A and B of different element codes (mixed fp8)."""
    a = np.ascontiguousarray(a)
    b = np.ascontiguousarray(b)
    m, k = a.shape
    n = b.shape[1]
    c = np.empty((m, n), np.float32)
    lib().oracle_gemm_mixed(dta, dtb, _p(a), _p(b), _p(c), m, n, k, threads)
    return c


def gemm_rows(dt: int, a, b, rows):
    """C rows for the given row indices only (sampled verification of big problems)."""
    a = np.ascontiguousarray(a[rows])
    return gemm(dt, a, b)


def count_abs_errors(got, ref, atol: float = 1e-2) -> int:
    got = np.ascontiguousarray(got, np.float32)
    ref = np.ascontiguousarray(ref, np.float32)
    return int(lib().oracle_count_abs_errors(_p(got), _p(ref), got.size, atol))


def prune_2of4(dt: int, a):
    a = np.ascontiguousarray(a)
    out = np.empty_like(a)
    lib().oracle_prune_2of4(dt, _p(a), a.shape[0], a.shape[1], _p(out))
    return out


def meta_tc_image(dt: int, meta, m: int, k: int):
    mb = ((m + 127) // 128 + 1) // 2 * 2
    ka = (k + 127) // 128
    img = np.empty(mb * ka * 512, np.uint32)
    lib().oracle_meta_tc_image(dt, _p(np.ascontiguousarray(meta)), m, k, _p(img))
    return img.view(np.uint8)


def quantize_e4m3(x):
    x = np.ascontiguousarray(x, np.float32)
    q = np.empty(x.shape, np.uint8)
    s = lib().oracle_quantize_e4m3(_p(x), x.size, _p(q))
    return q, float(s)


def quantize_e5m2(x):
    x = np.ascontiguousarray(x, np.float32)
    q = np.empty(x.shape, np.uint8)
    s = lib().oracle_quantize_e5m2(_p(x), x.size, _p(q))
    return q, float(s)


def to_float(dt: int, bits):
    bits = np.ascontiguousarray(bits)
    out = np.empty(bits.shape, np.float32)
    lib().oracle_to_float(dt, _p(bits), bits.size, _p(out))
    return out


def from_float(dt: int, x):
    x = np.ascontiguousarray(x, np.float32)
    out = np.empty(x.shape, BITS[dt])
    lib().oracle_from_float(dt, _p(x), x.size, _p(out))
    return out


def row_norm_rel_error(got, ref, a_f32, b_f32) -> float:
    """max |C - C_ref| / (||A[r,:]|| * ||B[:,n]|| / sqrt(K)) — the K-scaled
    row-norm relative error the parity bound is stated in."""
    k = a_f32.shape[1]
    denom = np.outer(np.linalg.norm(a_f32, axis=1), np.linalg.norm(b_f32, axis=0)) / np.sqrt(k)
    denom = np.maximum(denom, 1e-30)
    return float(np.max(np.abs(np.asarray(got, np.float32) - ref) / denom))


# ------------------------------------------------------------------ suites
_RAW_RE = re.compile(r"RawWgmmaSparseDemo<\s*([\w:]+)\s*,\s*(\d+)\s*>")
_CUTE_RE = re.compile(r"WgmmaSparseDemo<\s*([\w:]+)\s*,\s*[\w:]+\s*,.*?,\s*(\d+)\s*>\s*;", re.S)
_CASE_RE = re.compile(r'\{\s*"([^"]+)"\s*,\s*(\d+)\s*,\s*(\d+)\s*,\s*(\d+)\s*,\s*(true|false)\s*\}')
_RUNCASE_RE = re.compile(r'run_case\(\s*"([^"]+)"\s*,\s*(\d+)\s*,\s*(\d+)\s*,\s*(\d+)\s*,\s*(true|false)')


def parse_entry_point(path: str):
    """(harness, dtype, block_n, [(tag, m, n, k, pattern)]) of a reference main."""
    src = open(path).read()
    name = os.path.basename(path)
    m = _RAW_RE.search(src)
    if m:
        harness, dt, bn = "raw", NAMES[m.group(1)], int(m.group(2))
    else:
        m = _CUTE_RE.search(src)
        if m:
            harness, dt, bn = "cute", NAMES[m.group(1)], int(m.group(2))
        elif name == "mma_sp_wgmma_m64n8k32_fp32fp16.cu":
            harness, dt, bn = "cute_standalone", F16, 8
        else:
            return None
    cases = [(t, int(a), int(b), int(c), p == "true") for t, a, b, c, p in _CASE_RE.findall(src)]
    if not cases:
        cases = [(t, int(a), int(b), int(c), p == "true") for t, a, b, c, p in _RUNCASE_RE.findall(src)]
    return harness, dt, bn, cases
