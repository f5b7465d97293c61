import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a)")


@pytest.fixture(scope="session")
def cuda_device():
    """The GPU tests run only on a CUDA box; there they fail loudly if the native
    library or the device is missing (no CPU fallback exists)."""
    import torch
    if not torch.cuda.is_available():
        pytest.fail("GPU test run without a CUDA device")
    from mojollama_b200 import core
    lib = core()
    assert lib.mlq_init(0) == 0, lib.mlq_last_error_message()
    # launch on torch's current stream so device tensors written by torch are ordered
    assert lib.mlq_set_stream(torch.cuda.current_stream().cuda_stream) == 0
    return lib
