import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG = os.path.join(ROOT, "aicompiler-test_b200")
for p in (ROOT, PKG):
    if p not in sys.path:
        sys.path.insert(0, p)

GOLDEN = os.path.join(ROOT, "tests", "golden")


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100a) GPU")


@pytest.fixture(scope="session")
def rt():
    import tmc_cuda
    if tmc_cuda.device_count() == 0:
        pytest.fail("GPU test selected but no CUDA device is visible")
    runtime = tmc_cuda.Runtime(0)
    yield runtime
    runtime.close()
