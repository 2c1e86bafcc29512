"""The reference's own per-dtype entry points (mma_sp_wgmma_*.cu), compiled
unchanged against the drop-in headers and linked with libsp24, run on the
GPU: each must exit 0 after printing "Verification PASSED" (its three cases
checked with the reference's abs 1e-2 rule, after the GPU compression was
compared bit for bit with the host compression)."""
import os
import subprocess

import pytest

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
BIN = os.path.join(ROOT, "sparse-gemm-with-hopper-sptc_b200", "bin")
MAINS = sorted(m for m in os.listdir(BIN) if m.startswith("mma_sp_wgmma_")) if os.path.isdir(BIN) \
    else []


def test_all_entry_points_were_built():
    if not MAINS:
        pytest.skip("drop-in mains not built (no reference checkout at build time)")
    assert len([m for m in MAINS if m.startswith("mma_sp_wgmma_cuda_")]) == 18
    assert len([m for m in MAINS if not m.startswith("mma_sp_wgmma_cuda_")]) == 5


@pytest.mark.parametrize("main", MAINS)
def test_entry_point_passes(main):
    out = subprocess.run([os.path.join(BIN, main)], capture_output=True, text=True, timeout=300)
    assert out.returncode == 0, out.stdout + out.stderr
    assert "Verification PASSED" in out.stdout, out.stdout
    assert "total errors: 0" in out.stdout


@pytest.mark.parametrize("exe_name", ["raw_kernel_check", "raw_kernel_check_m128"])
def test_launchable_raw_kernel_matches_reference_cases(exe_name):
    """wgmma_sp_raw_kernel<Element, BlockN> of the drop-in, launched exactly as
    the reference's run_case launches its kernel (wgmma_sp_raw_common.hpp:
    1078-1080: grid (n / BlockN, m / 64), 128 threads, no dynamic shared
    memory), for all 18 (Element, BlockN) of the reference's raw entry points:
    each entry point's pattern and random cases plus a 320 x 3 BlockN grid,
    with the reference's host generation, compression, cpu_gemm_ref and abs
    1e-2 verify_result (tests/raw_kernel_check.cu).  Both forms: the default
    M = 64 MMA and the M = 128 MMA over zero-padded rows."""
    exe = os.path.join(BIN, exe_name)
    if not os.path.exists(exe):
        pytest.skip("raw_kernel_check not built")
    out = subprocess.run([exe], capture_output=True, text=True, timeout=600)
    assert out.returncode == 0, out.stdout[-4000:] + out.stderr[-2000:]
    assert "RAW KERNEL CHECK PASSED" in out.stdout
    assert out.stdout.count("total errors: 0") == 18 * 4
