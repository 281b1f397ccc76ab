import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG = os.path.join(ROOT, "apus-glm5.3-flash_b200")
for p in (ROOT, PKG, os.path.join(ROOT, "oracle")):
    if p not in sys.path:
        sys.path.insert(0, p)

GOLDEN = os.path.join(ROOT, "tests", "golden")


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100a) GPU")


@pytest.fixture(scope="session")
def gcuda():
    """The CUDA engine's C ABI, enabled on cuda:0 (GPU tests only)."""
    import torch
    assert torch.cuda.is_available(), "GPU test run without a GPU"
    torch.cuda.init()
    import apus_gcuda
    apus_gcuda.enable()
    return apus_gcuda
