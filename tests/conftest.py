"""Shared fixtures. GPU tests carry @pytest.mark.gpu; everything else runs on CPU."""
import os
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG = os.path.join(ROOT, "shannon-prime-system_b200")
ORACLE = os.path.join(ROOT, "oracle")
GOLDEN = os.path.join(ROOT, "tests", "golden")
for p in (PKG, ORACLE):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200) and the built libspb200.so")


@pytest.fixture(scope="session")
def xr():
    import xref
    if not os.path.exists(xref.XREF_SO):
        import subprocess
        subprocess.run(["make", "-C", ORACLE, "xref"], check=True, capture_output=True)
    return xref.Xref()


@pytest.fixture(scope="session")
def reflib():
    import xref
    if not os.path.exists(xref.SPREF_SO):
        pytest.skip("reference library oracle/_ref/libspref.so not built (reference tree absent)")
    import ctypes
    ctypes.CDLL(xref.SPREF_SO, mode=ctypes.RTLD_GLOBAL)
    return xref.RefLib()


@pytest.fixture(scope="session")
def spb():
    import spb200
    return spb200.load()


@pytest.fixture(scope="session")
def cuda_ok():
    import spb200
    L = spb200.load()
    if L.spb_device_count() < 1:
        pytest.fail("no CUDA device visible to libspb200.so")
    return True


def rng(seed):
    return np.random.default_rng(seed)
