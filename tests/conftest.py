import sys
from pathlib import Path

import pytest

REPO = Path(__file__).resolve().parents[1]
PKG_ROOT = REPO / "nanokv-llm_b200"
for p in (str(REPO), str(PKG_ROOT)):
    if p not in sys.path:
        sys.path.insert(0, p)

GOLDEN = REPO / "tests" / "golden"


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200, sm_100a)")


@pytest.fixture(scope="session")
def golden_dir():
    return GOLDEN


@pytest.fixture(scope="session")
def cuda_lib():
    """libnkv on a visible GPU; tests using it are marked gpu."""
    import torch

    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from nanokv_b200 import _lib

    lib = _lib.load()
    _lib.read_device_error(clear=True)
    return lib
