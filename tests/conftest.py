import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200, sm_100a)")


def gpu_available() -> bool:
    try:
        import torch
        return torch.cuda.is_available()
    except Exception:
        return False


@pytest.fixture(scope="session")
def cuda():
    """The GPU-test fixture: a B200 must be present and the library built.
    GPU tests fail (never fall back) when the CUDA library is missing."""
    import torch
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from bml_b200 import build
    build.build()
    import bml_b200._lib as L
    L.lib()
    return torch.device("cuda", 0)
