import os
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (sm_100a) and the built CUDA library")


import pytest  # noqa: E402


@pytest.fixture(params=["mma", "tc"])
def far_kernel(request):
    """Runs a test once with each far-read kernel (mma.sync tiles, tcgen05 tiles)."""
    from fold_b200 import kernels
    kernels.select_far_read_kernel(request.param)
    yield request.param
    kernels.select_far_read_kernel("auto")
