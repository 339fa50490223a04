import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100) GPU; run with -m gpu")


@pytest.fixture(scope="session")
def oracle():
    from oracle import oracle as o
    o.build()
    return o


@pytest.fixture(scope="session")
def golden_dir():
    return os.path.join(ROOT, "tests", "golden")


@pytest.fixture(scope="session")
def cuda():
    """The GEMM library on a CUDA device. A GPU test must not pass on a fallback: if the
    device or the native library is missing, this fails instead of skipping."""
    import torch
    if not torch.cuda.is_available():
        pytest.fail("GPU test selected but no CUDA device is visible")
    import hopper_gemm_b200 as hg
    cap = torch.cuda.get_device_capability(0)
    if cap != (10, 0):
        pytest.fail(f"expected an sm_100 device, found sm_{cap[0]}{cap[1]}")
    torch.cuda.init()
    return hg
