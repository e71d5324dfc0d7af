import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200, sm_100a)")


@pytest.fixture(scope="session", autouse=True)
def _native_library():
    """Make sure libmhc_b200.so exists (builds it with nvcc when missing/stale)."""
    from mhc_ascend_b200 import build
    if not build.up_to_date():
        try:
            build.build()
        except RuntimeError as e:  # no nvcc: the prebuilt library must be present
            if not os.path.exists(build.LIB_PATH):
                raise
            print("warning: could not rebuild libmhc_b200.so:", e)
    yield


@pytest.fixture
def cuda():
    import torch
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    return torch.device("cuda:0")
