import os
import subprocess
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
for p in (ROOT, os.path.join(ROOT, "bsscl-gbm_b200"), os.path.join(ROOT, "oracle")):
    if p not in sys.path:
        sys.path.insert(0, p)

GOLDEN = os.path.join(ROOT, "tests", "golden")
LIB = os.path.join(ROOT, "bsscl-gbm_b200", "bsscl_gbm_b200", "libgbm_b200.so")


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (NVIDIA B200)")


@pytest.fixture(scope="session")
def built_lib():
    """libgbm_b200.so, compiled with nvcc if it is missing (no GPU needed to build)."""
    if not os.path.exists(LIB):
        subprocess.run(["make", "-s", "-C", os.path.join(ROOT, "bsscl-gbm_b200", "csrc")], check=True)
    return LIB


@pytest.fixture(scope="session")
def engine():
    """One device context shared by the GPU tests."""
    from bsscl_gbm_b200 import Engine
    e = Engine(0)
    yield e
    e.close()
