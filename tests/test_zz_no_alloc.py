"""sp24_gemm_noalloc: the allocation-free GEMM entry point for callers that
may not allocate device memory per call (serving loops that forbid
cudaMalloc after start-up, since an allocation can synchronize the device;
plugin hosts that own all device memory and only hand over inputs and
outputs).  It stages its scratch in the library's fixed device
buffer instead of a caller workspace.

Checked through the C ABI against the regular sp24_gemm (which gets its own
workspace from the caller) on two consecutive calls with different data, so
the second call must not see stale scratch from the first.  The tests use
the same tolerances as the other parity tests: the reference's abs 1e-2 rule
against the CPU oracle, and equality with sp24_gemm (same kernels)."""
import ctypes

import numpy as np
import pytest
import torch

import oracle
import sp24

pytestmark = pytest.mark.gpu

DEV = torch.device("cuda:0")


def _to_dev(bits, dt):
    if bits.dtype == np.uint16:
        t = torch.from_numpy(np.ascontiguousarray(bits).view(np.int16))
        return t.view(torch.float16 if dt == 0 else torch.bfloat16).to(DEV)
    return torch.from_numpy(np.ascontiguousarray(bits)).to(DEV)


def _noalloc(ac, meta, b, m, n, k, dt):
    c = torch.full((m, n), float("nan"), device=DEV)
    d = sp24.make_desc(ac, meta, b, m, n, k, meta_format=sp24.META_REF, c_f32=c,
                       dtype={0: torch.float16, 1: torch.bfloat16, 2: torch.uint8}[dt])
    rc = sp24.load().sp24_gemm_noalloc(ctypes.byref(d), torch.cuda.current_stream().cuda_stream)
    assert rc == 0, sp24.STATUS.get(rc, rc)
    return c


@pytest.mark.parametrize("dt,shapes", [
    (1, [(256, 512, 1024), (512, 384, 512)]),     # reference metadata repacked into the buffer
    (2, [(64, 8, 256), (128, 16, 256)]),          # e4m3, n = 8: B also padded in the buffer
    (0, [(1024, 1024, 2048), (64, 128, 32)]),
])
def test_noalloc_matches_sp24_gemm_on_two_calls(dt, shapes):
    gen = oracle.Gen(77 + dt)
    for (m, n, k) in shapes:
        a, b, a_c, e, c_ref = oracle.host_case(gen, dt, m, n, k, False)
        ac_t, e_t = _to_dev(a_c, dt), _to_dev(e, dt)
        b_t = _to_dev(b, dt)
        c_noalloc = _noalloc(ac_t, e_t, b_t, m, n, k, dt)
        c_regular, _ = sp24.gemm(ac_t, e_t, b_t, m, n, k,
                                 dtype={0: torch.float16, 1: torch.bfloat16, 2: torch.uint8}[dt])
        torch.cuda.synchronize()
        assert sp24.last_kernel_status() == 0
        assert torch.equal(c_noalloc, c_regular)
        assert oracle.count_abs_errors(c_noalloc.cpu().numpy(), c_ref, 1e-2) == 0


def test_noalloc_rejects_problems_beyond_its_buffer():
    """An 8448 x 16384 A has a 17.3 MB metadata image, more than the 16 MiB
    buffer holds, so the call is refused before anything is launched."""
    m, k, n = 8448, 16384, 256
    assert sp24.meta_tc_bytes(m, k) > (16 << 20)
    d = sp24.GemmDesc()
    d.dtype, d.m, d.n, d.k = 1, m, n, k
    d.a_c, d.meta, d.b, d.c_f32 = 0x10000, 0x20000, 0x30000, 0x40000
    d.meta_format = sp24.META_REF
    assert sp24.load().sp24_gemm_noalloc(ctypes.byref(d), None) == 10


def _fake_desc(dt, m, n, k, meta_format, ldb=0):
    d = sp24.GemmDesc()
    d.dtype, d.m, d.n, d.k = dt, m, n, k
    d.a_c, d.meta, d.b, d.c_f32 = 0x10000, 0x20000, 0x30000, 0x40000
    d.meta_format, d.ldb = meta_format, ldb
    return d


def test_noalloc_counts_padded_b_toward_its_limit():
    """B whose row pitch breaks the 16-byte rule is staged padded in the same
    buffer, so its copy counts toward the limit: refused when the padded B
    alone is too large (tcgen05 metadata, nothing else in the buffer), and
    when metadata image plus padded B are too large although each would fit
    alone.  Host-side checks only: nothing is launched."""
    lib = sp24.load()
    limit = 16 << 20
    # 128 x 16384 bf16 A, B 16384 x 1001: padded pitch 1008 elements = 33 MB
    d = _fake_desc(1, 128, 1001, 16384, sp24.META_TC)
    assert sp24.workspace_bytes(d) > limit
    assert lib.sp24_gemm_noalloc(ctypes.byref(d), None) == 10
    # 4096 x 16384 A: 8.4 MB image; B 16384 x 301 (602 B rows): 9.96 MB padded
    d = _fake_desc(1, 4096, 301, 16384, sp24.META_REF)
    assert sp24.meta_tc_bytes(4096, 16384) < limit
    assert sp24.workspace_bytes(d) - sp24.meta_tc_bytes(4096, 16384) < limit
    assert sp24.workspace_bytes(d) > limit
    assert lib.sp24_gemm_noalloc(ctypes.byref(d), None) == 10


def test_noalloc_limit_boundary():
    """The largest documented fit: an 8192 x 16384 A's metadata image is
    exactly the 16 MiB buffer."""
    d = _fake_desc(1, 8192, 256, 16384, sp24.META_REF)
    assert sp24.workspace_bytes(d) == sp24.meta_tc_bytes(8192, 16384) == 16 << 20
