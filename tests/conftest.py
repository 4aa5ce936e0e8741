import os
import sys

import pytest

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if REPO not in sys.path:
    sys.path.insert(0, REPO)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 GPU (runs the CUDA library)")
    config.addinivalue_line("markers", "slow: multi-second CPU oracle work")


@pytest.fixture(scope="session", autouse=True)
def _native_build():
    """Builds the in-tree libraries if a source is newer than its build (no-op otherwise)."""
    from webgpu_b200 import build
    build.build_synth()
    build.build_oracle()
    build.build_cuda()
    yield


@pytest.fixture(scope="session")
def cuda():
    import torch
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    torch.cuda.init()
    return torch
