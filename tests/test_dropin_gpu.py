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
MAINS = sorted(os.listdir(BIN)) if os.path.isdir(BIN) else []


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
