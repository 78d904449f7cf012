import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200, sm_100a) and the built library")
    config.addinivalue_line("markers", "slow: long-running sweep")


def cuda_ok():
    try:
        import torch
        return torch.cuda.is_available()
    except Exception:
        return False


@pytest.fixture
def dev():
    if not cuda_ok():
        pytest.skip("requires a CUDA GPU")
    import torch
    return torch.device("cuda", torch.cuda.current_device())


@pytest.fixture(autouse=True)
def _device_status_clean(request):
    """After every GPU test the device status word must be clean (no expired
    wait, no failed index check)."""
    yield
    if request.node.get_closest_marker("gpu") is None or not cuda_ok():
        return
    from detkernels_b200 import _lib
    import torch
    code, detail = _lib.device_status(torch.cuda.current_device(), clear=True)
    assert code == 0, "device status %d detail 0x%x" % (code, detail)
