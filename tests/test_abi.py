"""The C ABI without a GPU: the library loads, exports every function
include/sp24.h declares, and rejects bad descriptors before touching CUDA."""
import ctypes
import os
import re
import subprocess

import pytest

import sp24

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "sp24.h")


def declared_functions():
    src = open(HEADER).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    return sorted(set(re.findall(r"\b(sp24_[a-z0-9_]+)\s*\(", src)))


def test_exports_every_declared_function():
    lib = sp24.load()
    names = declared_functions()
    assert len(names) >= 15
    for n in names:
        assert hasattr(lib, n), n
    assert set(names) <= set(sp24.EXPORTS) | {n for n in names if n in sp24.EXPORTS}


def test_loads_without_cuda_driver_dependency():
    out = subprocess.run(["ldd", sp24.LIB_PATH], capture_output=True, text=True).stdout
    assert "libcuda.so" not in out and "libtorch" not in out


def test_version_and_status_strings():
    lib = sp24.load()
    assert b"sm_100a" in lib.sp24_version()
    assert lib.sp24_status_string(0) == b"ok"
    assert b"2:4" in lib.sp24_status_string(3)


def test_meta_image_bytes():
    lib = sp24.load()
    assert lib.sp24_meta_tc_bytes(64, 32) == 2 * 2048          # one atom, padded to 2 blocks
    assert lib.sp24_meta_tc_bytes(8192, 8192) == 64 * 64 * 2048
    assert lib.sp24_meta_tc_bytes(129, 129) == 2 * 2 * 2048
    assert lib.sp24_meta_tc_bytes(0, 64) == 0


def _desc(**kw):
    base = dict(dtype=0, m=128, n=128, k=128, a_c=0x10000, lda_c=0, meta=0x20000,
                meta_format=sp24.META_TC, b=0x30000, ldb=0, c_f32=0x40000, c_bf16=0, ldc=0,
                alpha=1.0, tile_n=0, workspace=0, workspace_bytes=0, status_dev=0)
    base.update(kw)
    d = sp24.GemmDesc()
    for k, v in base.items():
        setattr(d, k, v)
    return d


@pytest.mark.parametrize("kw,code", [
    (dict(k=48), 1),                       # k % 32
    (dict(dtype=2, k=96), 1),              # e4m3 needs k % 64
    (dict(m=0), 1),
    (dict(a_c=0), 8),
    (dict(c_f32=0), 8),                    # no output at all
    (dict(dtype=7), 8),
    (dict(dtype=6), 8),                    # past the last mixed fp8 code
    (dict(dtype=3, k=96), 1),              # mixed fp8 (e5m2 x e4m3) needs k % 64
    (dict(dtype=4, k=32), 1),
    (dict(dtype=5, k=160), 1),
    (dict(a_c=0x10008), 2),                # A_c not 16-byte aligned
    (dict(lda_c=68), 2),                   # A_c row pitch not a multiple of 16 bytes
    (dict(lda_c=32), 1),                   # pitch smaller than k/2
    (dict(meta=0x20004), 2),
    (dict(tile_n=300), 8),
    (dict(meta_format=sp24.META_REF), 9),  # reference metadata needs a workspace
    (dict(meta_format=sp24.META_K16), 9),  # so does the m16n8k16 layout
    (dict(meta_format=sp24.META_K16, dtype=2, k=128), 1),   # 16-bit types only
    (dict(meta_format=sp24.META_K16, m=120), 1),            # whole 16-row blocks
    (dict(meta_format=3), 8),
])
def test_gemm_rejects_bad_descriptors_before_cuda(kw, code):
    lib = sp24.load()
    assert lib.sp24_gemm(ctypes.byref(_desc(**kw)), None) == code
    assert lib.sp24_gemm(None, None) == 8


def test_workspace_sizes():
    assert sp24.workspace_bytes(_desc()) == 0
    assert sp24.workspace_bytes(_desc(meta_format=sp24.META_REF)) == 2 * 2048
    # e4m3 with n = 8: the row pitch of B (8 bytes) breaks the TMA 16-byte rule,
    # so B is staged into a padded copy (pitch 16) inside the workspace.
    need = sp24.workspace_bytes(_desc(dtype=2, n=8, meta_format=sp24.META_REF))
    assert need == 2 * 2048 + 16 * 128


@pytest.mark.parametrize("n,world,align", [(65536, 8, 256), (1000, 3, 256), (20, 4, 16),
                                           (8192, 2, 256), (257, 2, 256)])
def test_shard_columns_partition(n, world, align):
    spans = [sp24.shard_columns(n, world, r, align) for r in range(world)]
    assert spans[0][0] == 0 and spans[-1][1] == n
    for (a0, a1), (b0, b1) in zip(spans, spans[1:]):
        assert a1 == b0 and a0 <= a1
    for a0, _ in spans:
        assert a0 % align == 0 or a0 == n


def test_compress_and_prune_argument_checks():
    lib = sp24.load()
    bad = ctypes.c_longlong(0)
    assert lib.sp24_compress(0, None, 8, 8, 0, None, 0, None, None, ctypes.byref(bad), None) == 8
    assert lib.sp24_compress(0, 0x1000, 8, 12, 0, 0x2000, 0, 0x3000, 0x4000, None, None) == 1
    assert lib.sp24_compress(0, 0x1008, 8, 16, 0, 0x2000, 0, 0x3000, 0x4000, None, None) == 2
    assert lib.sp24_prune_2of4(0, 0x1000, 8, 6, 0, 0x2000, 0, None) == 1
    assert lib.sp24_repack_meta(0, 0x1000, 64, 48, 0x2000, None) == 1


def _multi(**kw):
    md = sp24.MultiDesc()
    md.gemm.dtype, md.gemm.m, md.gemm.n, md.gemm.k = 1, 256, 512, 256
    md.gemm.meta_format = sp24.META_TC
    md.ngpu = kw.pop("ngpu", 2)
    for g in range(min(md.ngpu, sp24.MAX_GPUS)):
        md.devices[g] = g
        md.a_c[g], md.meta[g], md.b[g] = 0x10000, 0x20000, 0x30000
        md.c_f32[g] = 0x40000
    for k, v in kw.items():
        setattr(md, k, v)
    return md


def test_gemm_multi_rejects_bad_descriptors_before_any_launch():
    """sp24_gemm_multi's structural checks run on the host before any CUDA
    call: GPU count, repeated devices, layouts, missing pointers, and an
    all-gather into column-block (SHARD) outputs."""
    lib = sp24.load()
    call = lambda md, ag=0: lib.sp24_gemm_multi(ctypes.byref(md), ag)
    assert call(_multi(ngpu=0)) == 8
    assert call(_multi(ngpu=9)) == 8
    md = _multi()
    md.devices[1] = 0
    assert call(md) == 8
    md = _multi()
    md.b[1] = None
    assert call(md) == 8
    md = _multi()
    md.c_f32[1] = None                       # outputs must match across devices
    assert call(md) == 8
    assert call(_multi(c_layout=sp24.MULTI_SHARD), 1) == 8
    assert call(_multi(b_layout=7)) == 8
    md = _multi()
    md.gemm.k = 48                           # k % 32 for 16-bit types
    assert call(md) == 1
    md = _multi()
    md.gemm.ldc = 300                        # a whole-matrix C must span all 512 columns
    assert call(md) == 1
    md = _multi()
    md.gemm.ldb = 300
    assert call(md) == 1
    md = _multi(b_layout=sp24.MULTI_SHARD, c_layout=sp24.MULTI_SHARD)
    md.gemm.ldc = md.gemm.ldb = 300          # column-block layouts use their own widths
    assert lib.sp24_gemm_multi_workspace_bytes(ctypes.byref(md)) == 0
    assert lib.sp24_replicate(None, 0, 16, 1, None, None, None) == 8
    assert lib.sp24_gemm_multi_workspace_bytes(ctypes.byref(_multi(ngpu=0))) == 0
    md = _multi()
    md.gemm.n = 700                          # 188-column second block: B padded in workspace
    md.b_layout = sp24.MULTI_SHARD
    assert lib.sp24_gemm_multi_workspace_bytes(ctypes.byref(md)) == 256 * 384
