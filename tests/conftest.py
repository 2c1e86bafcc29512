"""Shared test setup.  Tests marked `gpu` need a B200 (sm_100); everything
else runs on the CPU.  The built libraries are produced in-tree by
__graft_entry__.build(); the session fixture rebuilds only what is stale."""
import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG = os.path.join(ROOT, "sparse-gemm-with-hopper-sptc_b200")
for p in (PKG, os.path.join(ROOT, "oracle"), ROOT):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs an sm_100 (B200) GPU")


@pytest.fixture(scope="session", autouse=True)
def _built():
    import build as sp24_build
    sp24_build.build_lib()
    if not os.path.exists(os.path.join(ROOT, "oracle", "lib", "libsp24_oracle.so")):
        sp24_build.build_oracle()
    yield


@pytest.fixture(scope="session")
def golden():
    import json
    import numpy as np
    d = os.path.join(ROOT, "tests", "golden")
    meta = json.load(open(os.path.join(d, "golden.json")))
    arrays = np.load(os.path.join(d, "golden.npz"))
    return meta, arrays
