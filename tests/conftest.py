import os
import sys

import pytest

sys.path.insert(0, os.path.dirname(os.path.abspath(__file__)))
# the package binding (veltrix-engine_b200/vxb200.py), for tests run on their own
sys.path.insert(0, os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "veltrix-engine_b200"))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a)")
    config.addinivalue_line("markers", "slow: longer CPU test")


@pytest.fixture(scope="session")
def cuda():
    """torch with a CUDA device, and the library initialised on device 0."""
    import torch
    if not torch.cuda.is_available():
        pytest.fail("this test needs a CUDA device")
    import vxb200
    vxb200.check(vxb200.lib().vxc_device_init(0), "vxc_device_init")
    return torch
