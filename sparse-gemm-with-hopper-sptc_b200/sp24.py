"""ctypes binding of the sp24 C ABI (include/sp24.h) for tests and the bench.

The product is the C-ABI shared library ``lib/libsp24.so`` built from
``csrc/`` for sm_100a.  This module only marshals torch CUDA tensors into the
plain pointers/sizes that ABI takes; every computation runs in the library's
CUDA kernels.  There is no CPU path: if the library or a GPU is missing, the
calls raise.

Reference interfaces mirrored (codes1gn/sparse-gemm-with-hopper-sptc):
  gemm()      wgmma_sp_raw_kernel<Element,BlockN>, wgmma_sp_raw_common.hpp:955-1030
  compress()  compress_structured_sparse_a, wgmma_sp_raw_common.hpp:140-205
"""
from __future__ import annotations

import ctypes
import os
from ctypes import (POINTER, Structure, c_char_p, c_float, c_int, c_int64, c_longlong,
                    c_size_t, c_uint8, c_ulonglong, c_void_p)

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "lib", "libsp24.so")
PEAK_LIB_PATH = os.path.join(HERE, "lib", "libsp24_peak.so")

F16, BF16, E4M3 = 0, 1, 2
# Mixed fp8: A's format first, B's second (kind::f8f6f4 formats may differ).
E5M2_E4M3, E4M3_E5M2, E5M2 = 3, 4, 5
META_REF, META_TC, META_K16 = 0, 1, 2

STATUS = {
    0: "SP24_OK", 1: "SP24_ERR_SHAPE", 2: "SP24_ERR_ALIGN", 3: "SP24_ERR_NOT_2OF4",
    4: "SP24_ERR_ARCH", 5: "SP24_ERR_CUDA", 6: "SP24_ERR_TIMEOUT", 7: "SP24_ERR_NCCL",
    8: "SP24_ERR_ARG", 9: "SP24_ERR_WORKSPACE", 10: "SP24_ERR_SCRATCH_LIMIT",
}

# Every symbol include/sp24.h declares.
EXPORTS = [
    "sp24_version", "sp24_status_string", "sp24_check_device", "sp24_meta_tc_bytes",
    "sp24_gemm_workspace_bytes", "sp24_compress", "sp24_prune_2of4", "sp24_repack_meta",
    "sp24_gemm", "sp24_last_kernel_status", "sp24_selftest_timeout", "sp24_amax_f32",
    "sp24_quantize_e4m3", "sp24_shard_columns", "sp24_unshard_columns_f32",
    "sp24_gemm_noalloc", "sp24_quantize_e5m2", "sp24_gemm_fused", "sp24_repack_meta_k16",
    "sp24_gemm_allgather", "sp24_ipc_get_handle", "sp24_ipc_open_handle", "sp24_ipc_close",
    "sp24_set_launch_hints", "sp24_get_launch_hints", "sp24_reload_tuning",
    "sp24_gemm_multi", "sp24_replicate", "sp24_gemm_multi_workspace_bytes",
]
MAX_PEERS = 7
HINT_NONE, HINT_STATIC_WEIGHTS = 0, 1

ACT_NONE, ACT_SILU = 0, 1


class Sp24Error(RuntimeError):
    def __init__(self, code: int, where: str):
        self.code = code
        super().__init__(f"{where}: {STATUS.get(code, code)}")


class GemmDesc(Structure):
    _fields_ = [
        ("dtype", c_int), ("m", c_int), ("n", c_int), ("k", c_int),
        ("a_c", c_void_p), ("lda_c", c_int64),
        ("meta", c_void_p), ("meta_format", c_int),
        ("b", c_void_p), ("ldb", c_int64),
        ("c_f32", c_void_p), ("c_bf16", c_void_p), ("ldc", c_int64),
        ("alpha", c_float), ("tile_n", c_int),
        ("workspace", c_void_p), ("workspace_bytes", c_size_t),
        ("status_dev", c_void_p),
    ]


class Epilogue(Structure):
    _fields_ = [
        ("bias", c_void_p), ("act", c_int),
        ("a_c_up", c_void_p), ("lda_c_up", c_int64), ("meta_up", c_void_p),
        ("alpha_up", c_float), ("bias_up", c_void_p),
    ]


class PeerOut(Structure):
    _fields_ = [("n_peers", c_int), ("c_f32", c_void_p * 7), ("c_bf16", c_void_p * 7)]


MAX_GPUS = 8
MULTI_FULL, MULTI_SHARD = 0, 1


class MultiDesc(Structure):
    _fields_ = [
        ("gemm", GemmDesc), ("ngpu", c_int), ("devices", c_int * MAX_GPUS),
        ("streams", c_void_p * MAX_GPUS), ("a_c", c_void_p * MAX_GPUS),
        ("meta", c_void_p * MAX_GPUS), ("b", c_void_p * MAX_GPUS), ("b_layout", c_int),
        ("c_f32", c_void_p * MAX_GPUS), ("c_bf16", c_void_p * MAX_GPUS), ("c_layout", c_int),
        ("workspace", c_void_p * MAX_GPUS), ("workspace_bytes", c_size_t),
    ]


_lib = None


def load(path: str = LIB_PATH) -> ctypes.CDLL:
    """Load the shared library (raises if it was not built)."""
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(path):
        raise FileNotFoundError(f"{path} missing: run __graft_entry__.build() first")
    lib = ctypes.CDLL(path)
    lib.sp24_version.restype = c_char_p
    lib.sp24_status_string.restype = c_char_p
    lib.sp24_status_string.argtypes = [c_int]
    lib.sp24_check_device.argtypes = [c_int]
    lib.sp24_meta_tc_bytes.restype = c_size_t
    lib.sp24_meta_tc_bytes.argtypes = [c_int, c_int]
    lib.sp24_gemm_workspace_bytes.restype = c_size_t
    lib.sp24_gemm_workspace_bytes.argtypes = [POINTER(GemmDesc)]
    lib.sp24_gemm.argtypes = [POINTER(GemmDesc), c_void_p]
    lib.sp24_gemm_noalloc.argtypes = [POINTER(GemmDesc), c_void_p]
    lib.sp24_gemm_fused.argtypes = [POINTER(GemmDesc), POINTER(Epilogue), c_void_p]
    lib.sp24_gemm_allgather.argtypes = [POINTER(GemmDesc), POINTER(PeerOut), c_void_p]
    lib.sp24_gemm_multi.argtypes = [POINTER(MultiDesc), c_int]
    lib.sp24_gemm_multi_workspace_bytes.argtypes = [POINTER(MultiDesc)]
    lib.sp24_gemm_multi_workspace_bytes.restype = c_size_t
    lib.sp24_replicate.argtypes = [c_void_p, c_int, c_size_t, c_int, POINTER(c_int),
                                   POINTER(c_void_p), POINTER(c_void_p)]
    lib.sp24_ipc_get_handle.argtypes = [c_void_p, c_void_p, POINTER(c_size_t)]
    lib.sp24_ipc_open_handle.argtypes = [c_void_p, POINTER(c_void_p)]
    lib.sp24_ipc_close.argtypes = [c_void_p]
    lib.sp24_selftest_timeout.argtypes = [POINTER(GemmDesc), c_ulonglong, c_void_p]
    lib.sp24_last_kernel_status.argtypes = [c_void_p]
    lib.sp24_set_launch_hints.argtypes = [ctypes.c_uint]
    lib.sp24_set_launch_hints.restype = None
    lib.sp24_get_launch_hints.restype = ctypes.c_uint
    lib.sp24_reload_tuning.restype = None
    lib.sp24_reload_tuning.argtypes = []
    lib.sp24_compress.argtypes = [c_int, c_void_p, c_int, c_int, c_int64, c_void_p, c_int64,
                                  c_void_p, c_void_p, POINTER(c_longlong), c_void_p]
    lib.sp24_prune_2of4.argtypes = [c_int, c_void_p, c_int, c_int, c_int64, c_void_p, c_int64,
                                    c_void_p]
    lib.sp24_repack_meta.argtypes = [c_int, c_void_p, c_int, c_int, c_void_p, c_void_p]
    lib.sp24_repack_meta_k16.argtypes = [c_int, c_void_p, c_int, c_int, c_void_p, c_void_p]
    lib.sp24_amax_f32.argtypes = [c_void_p, c_size_t, c_void_p, c_void_p]
    lib.sp24_quantize_e4m3.argtypes = [c_void_p, c_size_t, c_void_p, c_void_p, c_void_p,
                                       c_void_p]
    lib.sp24_quantize_e5m2.argtypes = [c_void_p, c_size_t, c_void_p, c_void_p, c_void_p,
                                       c_void_p]
    lib.sp24_shard_columns.restype = None
    lib.sp24_shard_columns.argtypes = [c_int, c_int, c_int, c_int, POINTER(c_int),
                                       POINTER(c_int)]
    lib.sp24_unshard_columns_f32.argtypes = [c_void_p, c_void_p, c_int, c_int, c_int, c_int,
                                             c_void_p]
    for name in ("sp24_gemm", "sp24_gemm_noalloc", "sp24_gemm_fused", "sp24_gemm_allgather",
                 "sp24_gemm_multi", "sp24_replicate",
                 "sp24_ipc_get_handle", "sp24_ipc_open_handle", "sp24_ipc_close",
                 "sp24_selftest_timeout",
                 "sp24_last_kernel_status",
                 "sp24_compress", "sp24_prune_2of4", "sp24_repack_meta", "sp24_repack_meta_k16",
                 "sp24_amax_f32",
                 "sp24_quantize_e4m3", "sp24_quantize_e5m2", "sp24_unshard_columns_f32",
                 "sp24_check_device"):
        getattr(lib, name).restype = c_int
    _lib = lib
    return lib


def _check(code: int, where: str) -> None:
    if code != 0:
        raise Sp24Error(code, where)


def _ptr(t) -> int:
    return 0 if t is None else t.data_ptr()


def _stream(stream) -> int:
    import torch
    if stream is None:
        stream = torch.cuda.current_stream()
    return stream.cuda_stream


def dtype_code(tdtype) -> int:
    """Library dtype of a torch dtype (uint8 = e4m3 bits); ints pass through
    (the mixed fp8 codes cannot be told from one tensor)."""
    import torch
    if isinstance(tdtype, int):
        return tdtype
    if tdtype == torch.float8_e5m2:
        return E5M2
    if tdtype == torch.float16:
        return F16
    if tdtype == torch.bfloat16:
        return BF16
    if tdtype in (torch.float8_e4m3fn, torch.uint8):
        return E4M3
    raise ValueError(f"unsupported dtype {tdtype}")


def meta_tc_bytes(m: int, k: int) -> int:
    return int(load().sp24_meta_tc_bytes(m, k))


def compress(a_dense, stream=None, dtype=None):
    """Dense 2:4 A (m x k, CUDA) -> (A_c m x k/2, reference metadata m x k/8 uint8).
    dtype: library dtype code when the tensor's own dtype does not say it
    (fp8 bits held as uint8)."""
    import torch
    lib = load()
    m, k = a_dense.shape
    a_c = torch.empty((m, k // 2), dtype=a_dense.dtype, device=a_dense.device)
    meta = torch.empty((m, k // 8), dtype=torch.uint8, device=a_dense.device)
    bad_dev = torch.empty(1, dtype=torch.int64, device=a_dense.device)
    bad = c_longlong(-1)
    code = lib.sp24_compress(dtype_code(dtype if dtype is not None else a_dense.dtype),
                             _ptr(a_dense), m, k, a_dense.stride(0),
                             _ptr(a_c), a_c.stride(0), _ptr(meta), _ptr(bad_dev),
                             ctypes.byref(bad), _stream(stream))
    if code == 3:
        err = Sp24Error(code, f"sp24_compress (first bad group {bad.value})")
        err.bad_group = bad.value
        raise err
    _check(code, "sp24_compress")
    return a_c, meta


def prune_2of4(a, stream=None, dtype=None):
    import torch
    lib = load()
    m, k = a.shape
    out = torch.empty_like(a)
    code = dtype_code(dtype if dtype is not None else a.dtype)
    _check(lib.sp24_prune_2of4(code, _ptr(a), m, k, a.stride(0), _ptr(out),
                               out.stride(0), _stream(stream)), "sp24_prune_2of4")
    return out


def repack_meta(meta_ref, m: int, k: int, dtype, stream=None):
    import torch
    lib = load()
    out = torch.empty(meta_tc_bytes(m, k), dtype=torch.uint8, device=meta_ref.device)
    _check(lib.sp24_repack_meta(dtype_code(dtype), _ptr(meta_ref), m, k, _ptr(out),
                                _stream(stream)), "sp24_repack_meta")
    return out


def repack_meta_k16(meta_k16, m: int, k: int, dtype, stream=None):
    """tcgen05 image from metadata in the reference's m16n8k16 layout."""
    import torch
    lib = load()
    out = torch.empty(meta_tc_bytes(m, k), dtype=torch.uint8, device=meta_k16.device)
    _check(lib.sp24_repack_meta_k16(dtype_code(dtype), _ptr(meta_k16), m, k, _ptr(out),
                                    _stream(stream)), "sp24_repack_meta_k16")
    return out


def make_desc(a_c, meta, b, m, n, k, *, meta_format=META_REF, c_f32=None, c_bf16=None,
              alpha=1.0, tile_n=0, workspace=None, status=None, dtype=None) -> GemmDesc:
    d = GemmDesc()
    d.dtype = dtype_code(dtype if dtype is not None else a_c.dtype)
    d.m, d.n, d.k = m, n, k
    d.a_c, d.lda_c = _ptr(a_c), a_c.stride(0)
    d.meta, d.meta_format = _ptr(meta), meta_format
    d.b, d.ldb = _ptr(b), b.stride(0)
    d.c_f32, d.c_bf16 = _ptr(c_f32), _ptr(c_bf16)
    ref = c_f32 if c_f32 is not None else c_bf16
    d.ldc = ref.stride(0)
    d.alpha = alpha
    d.tile_n = tile_n
    d.workspace = _ptr(workspace)
    d.workspace_bytes = 0 if workspace is None else workspace.numel() * workspace.element_size()
    d.status_dev = _ptr(status)
    return d


def workspace_bytes(desc: GemmDesc) -> int:
    return int(load().sp24_gemm_workspace_bytes(ctypes.byref(desc)))


def gemm(a_c, meta, b, m, n, k, *, meta_format=META_REF, out_f32=True, out_bf16=False,
         alpha=1.0, tile_n=0, workspace=None, c_f32=None, c_bf16=None, stream=None,
         dtype=None):
    """C = alpha * decompress(A_c, meta) @ B through sp24_gemm.  Returns (c_f32, c_bf16)."""
    import torch
    lib = load()
    dev = a_c.device
    if out_f32 and c_f32 is None:
        c_f32 = torch.empty((m, n), dtype=torch.float32, device=dev)
    if out_bf16 and c_bf16 is None:
        c_bf16 = torch.empty((m, n), dtype=torch.bfloat16, device=dev)
    d = make_desc(a_c, meta, b, m, n, k, meta_format=meta_format, c_f32=c_f32, c_bf16=c_bf16,
                  alpha=alpha, tile_n=tile_n, workspace=workspace, dtype=dtype)
    need = workspace_bytes(d)
    if need and (workspace is None or d.workspace_bytes < need):
        workspace = torch.empty(need, dtype=torch.uint8, device=dev)
        d.workspace, d.workspace_bytes = workspace.data_ptr(), need
    _check(lib.sp24_gemm(ctypes.byref(d), _stream(stream)), "sp24_gemm")
    return c_f32, c_bf16


def gemm_fused(a_c, meta, b, m, n, k, *, bias=None, act=ACT_NONE, a_c_up=None, meta_up=None,
               alpha_up=1.0, bias_up=None, meta_format=META_TC, out_f32=True, out_bf16=False,
               alpha=1.0, tile_n=0, c_f32=None, c_bf16=None, stream=None, dtype=None):
    """sp24_gemm_fused: C = act(alpha A B + bias) [* (alpha_up A_up B + bias_up)]."""
    import torch
    lib = load()
    dev = a_c.device
    if out_f32 and c_f32 is None:
        c_f32 = torch.empty((m, n), dtype=torch.float32, device=dev)
    if out_bf16 and c_bf16 is None:
        c_bf16 = torch.empty((m, n), dtype=torch.bfloat16, device=dev)
    d = make_desc(a_c, meta, b, m, n, k, meta_format=meta_format, c_f32=c_f32, c_bf16=c_bf16,
                  alpha=alpha, tile_n=tile_n, dtype=dtype)
    need = workspace_bytes(d)
    ws = None
    if need:
        ws = torch.empty(need, dtype=torch.uint8, device=dev)
        d.workspace, d.workspace_bytes = ws.data_ptr(), need
    e = Epilogue()
    e.bias, e.act = _ptr(bias), act
    e.a_c_up = _ptr(a_c_up)
    e.lda_c_up = 0 if a_c_up is None else a_c_up.stride(0)
    e.meta_up, e.alpha_up, e.bias_up = _ptr(meta_up), alpha_up, _ptr(bias_up)
    _check(lib.sp24_gemm_fused(ctypes.byref(d), ctypes.byref(e), _stream(stream)),
           "sp24_gemm_fused")
    return c_f32, c_bf16


def ipc_handle(t):
    """(64-byte handle, byte offset) of the CUDA allocation holding tensor t."""
    h = ctypes.create_string_buffer(64)
    off = c_size_t(0)
    _check(load().sp24_ipc_get_handle(_ptr(t), h, ctypes.byref(off)), "sp24_ipc_get_handle")
    return h.raw, off.value


def ipc_open(handle: bytes) -> int:
    """Map a peer's allocation into this process; returns its base address."""
    base = c_void_p(0)
    buf = ctypes.create_string_buffer(handle, 64)
    _check(load().sp24_ipc_open_handle(buf, ctypes.byref(base)), "sp24_ipc_open_handle")
    return base.value


def ipc_close(base: int) -> None:
    _check(load().sp24_ipc_close(c_void_p(base)), "sp24_ipc_close")


def gemm_allgather(desc: GemmDesc, peer_f32=(), peer_bf16=(), stream=None) -> None:
    """sp24_gemm_allgather with peer element addresses (ints) for each output."""
    po = PeerOut()
    po.n_peers = max(len(peer_f32), len(peer_bf16))
    for i, a in enumerate(peer_f32):
        po.c_f32[i] = a
    for i, a in enumerate(peer_bf16):
        po.c_bf16[i] = a
    _check(load().sp24_gemm_allgather(ctypes.byref(desc), ctypes.byref(po), _stream(stream)),
           "sp24_gemm_allgather")


def replicate(src, dsts, streams=None) -> None:
    """sp24_replicate: copy tensor src into each tensor of dsts (one per
    device, same size), enqueued on each destination device's stream."""
    n = len(dsts)
    devs = (c_int * n)(*[t.device.index for t in dsts])
    ptrs = (c_void_p * n)(*[t.data_ptr() for t in dsts])
    strs = (c_void_p * n)(*[(s.cuda_stream if s is not None else None) for s in
                            (streams or [None] * n)])
    _check(load().sp24_replicate(src.data_ptr(), src.device.index,
                                 src.numel() * src.element_size(), n, devs, ptrs, strs),
           "sp24_replicate")


def make_multi_desc(m, n, k, dtype, a_c, meta, b, *, c_f32=None, c_bf16=None,
                    meta_format=META_TC, b_layout=MULTI_FULL, c_layout=MULTI_FULL, ldb=0, ldc=0,
                    alpha=1.0, workspaces=None, streams=None) -> MultiDesc:
    """A sp24_multi_desc from per-device tensors (lists, one per GPU, in
    device order)."""
    md = MultiDesc()
    g = md.gemm
    g.dtype, g.m, g.n, g.k = dtype_code(dtype), m, n, k
    g.meta_format, g.ldb, g.ldc, g.alpha = meta_format, ldb, ldc, alpha
    md.ngpu = len(a_c)
    for i, t in enumerate(a_c):
        md.devices[i] = t.device.index
        md.a_c[i], md.meta[i], md.b[i] = t.data_ptr(), meta[i].data_ptr(), b[i].data_ptr()
        md.c_f32[i] = _ptr(c_f32[i]) if c_f32 is not None else None
        md.c_bf16[i] = _ptr(c_bf16[i]) if c_bf16 is not None else None
        md.streams[i] = streams[i].cuda_stream if streams is not None else None
        if workspaces is not None and workspaces[i] is not None:
            md.workspace[i] = workspaces[i].data_ptr()
    if workspaces is not None:
        md.workspace_bytes = min(w.numel() for w in workspaces if w is not None)
    md.b_layout, md.c_layout = b_layout, c_layout
    g.lda_c = a_c[0].stride(0)
    return md


def multi_workspace_bytes(md: MultiDesc) -> int:
    return int(load().sp24_gemm_multi_workspace_bytes(ctypes.byref(md)))


def gemm_multi(md: MultiDesc, allgather_c: bool = False) -> list:
    """sp24_gemm_multi; when md carries no workspaces and the problem needs
    them, allocates one per device first.  Returns the workspaces (keep them
    alive until the streams are done)."""
    import torch
    keep = []
    need = multi_workspace_bytes(md)
    if need and not any(md.workspace[i] for i in range(md.ngpu)):
        for i in range(md.ngpu):
            w = torch.empty(need, dtype=torch.uint8, device=torch.device("cuda", md.devices[i]))
            md.workspace[i] = w.data_ptr()
            keep.append(w)
        md.workspace_bytes = need
    _check(load().sp24_gemm_multi(ctypes.byref(md), 1 if allgather_c else 0), "sp24_gemm_multi")
    return keep


def set_launch_hints(hints: int) -> None:
    """sp24_set_launch_hints for later GEMM calls of this thread
    (HINT_STATIC_WEIGHTS: A_c / metadata images are not written by in-flight work)."""
    load().sp24_set_launch_hints(hints)


def get_launch_hints() -> int:
    return load().sp24_get_launch_hints()


def reload_tuning() -> None:
    """sp24_reload_tuning: the library reads its SP24_* tuning variables once;
    call this after changing them in os.environ."""
    load().sp24_reload_tuning()


class tuning_env:
    """Context manager: set SP24_* tuning variables for the calls inside it
    (and re-read them in the library), restoring the old values on exit."""

    def __init__(self, env: dict):
        self.env = {k: str(v) for k, v in env.items()}

    def __enter__(self):
        self.old = {k: os.environ.get(k) for k in self.env}
        os.environ.update(self.env)
        reload_tuning()
        return self

    def __exit__(self, *exc):
        for k, v in self.old.items():
            if v is None:
                os.environ.pop(k, None)
            else:
                os.environ[k] = v
        reload_tuning()


def last_kernel_status(stream=None) -> int:
    return int(load().sp24_last_kernel_status(_stream(stream)))


def amax_quantize_e4m3(x, stream=None, e5m2=False):
    """fp32 CUDA tensor -> (fp8 bits as uint8, scale tensor[1]) with scale =
    448/amax (e4m3) or 57344/amax (e5m2)."""
    import torch
    lib = load()
    amax = torch.empty(1, dtype=torch.float32, device=x.device)
    scale = torch.empty(1, dtype=torch.float32, device=x.device)
    q = torch.empty(x.shape, dtype=torch.uint8, device=x.device)
    s = _stream(stream)
    _check(lib.sp24_amax_f32(_ptr(x), x.numel(), _ptr(amax), s), "sp24_amax_f32")
    fn = lib.sp24_quantize_e5m2 if e5m2 else lib.sp24_quantize_e4m3
    _check(fn(_ptr(x), x.numel(), _ptr(amax), _ptr(scale), _ptr(q), s),
           "sp24_quantize_e5m2" if e5m2 else "sp24_quantize_e4m3")
    return q, scale


def amax_quantize_e5m2(x, stream=None):
    return amax_quantize_e4m3(x, stream, e5m2=True)


def shard_columns(n: int, world: int, rank: int, align: int):
    a, b = c_int(0), c_int(0)
    load().sp24_shard_columns(n, world, rank, align, ctypes.byref(a), ctypes.byref(b))
    return a.value, b.value


def unshard_columns_f32(src, m: int, n: int, world: int, align: int, stream=None):
    import torch
    dst = torch.empty((m, n), dtype=torch.float32, device=src.device)
    _check(load().sp24_unshard_columns_f32(_ptr(src), _ptr(dst), m, n, world, align,
                                           _stream(stream)), "sp24_unshard_columns_f32")
    return dst


_peak = None


def probe_mma_rate(dtype: int, sparse: bool, iters: int = 4096, reps: int = 5, stream=None):
    """Tensor-core rate of the CTA-pair MMA shape with operands resident in
    shared memory (lib/libsp24_peak.so, measurement only): returns
    (dense-equivalent TFLOP/s, ms per launch).  dtype: F16, BF16 or E4M3."""
    global _peak
    import torch
    if _peak is None:
        if not os.path.exists(PEAK_LIB_PATH):
            raise FileNotFoundError(f"{PEAK_LIB_PATH} missing: run __graft_entry__.build() first")
        _peak = ctypes.CDLL(PEAK_LIB_PATH)
        _peak.sp24_probe_mma_rate.restype = c_int
        _peak.sp24_probe_mma_rate.argtypes = [c_int, c_int, c_int, c_int, POINTER(c_float),
                                              POINTER(ctypes.c_double), c_void_p, c_void_p]
    ms, flops = c_float(0.0), ctypes.c_double(0.0)
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    _check(_peak.sp24_probe_mma_rate(dtype, 1 if sparse else 0, iters, reps, ctypes.byref(ms),
                                     ctypes.byref(flops), _ptr(status), _stream(stream)),
           "sp24_probe_mma_rate")
    torch.cuda.synchronize()
    if status.item() != 0:
        raise Sp24Error(6, "sp24_probe_mma_rate")
    return flops.value / (ms.value * 1e-3) / 1e12, ms.value
