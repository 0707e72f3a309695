import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device of compute capability 10.x (B200)")


@pytest.fixture(scope="session")
def native_lib():
    """libms_cuda_nbits.so, built in-tree if missing (nvcc cross-compiles without a GPU)."""
    from modelsharp_b200 import _native, build
    if not _native.library_path().exists():
        build.build()
    return _native.lib()


@pytest.fixture(scope="session")
def cuda_device():
    import torch
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from modelsharp_b200 import _native
    assert _native.available(), "CUDA device present but not compute capability 10.x"
    return torch.device("cuda", 0)
