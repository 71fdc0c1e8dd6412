import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100a) and the built CUDA library")


@pytest.fixture(scope="session")
def cuda_lib():
    """The CUDA C-ABI library; GPU tests fail loudly (not skip) when it is missing."""
    import torch

    if not torch.cuda.is_available():
        pytest.fail("GPU test selected but CUDA is unavailable")
    from oscar_new_b200 import _lib

    return _lib.lib()
