import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200) and the built libes_moe.so")


def pytest_collection_modifyitems(config, items):
    """GPU tests fail loudly (not skip) when a GPU was asked for but is absent;
    when the run deselects them with -m "not gpu" they never reach here."""
    return


@pytest.fixture(scope="session")
def cuda():
    import torch
    if not torch.cuda.is_available():
        pytest.fail("this test needs a CUDA device")
    from expert_sniper_b200 import _native
    _native.lib()  # raises if the library is missing: no silent fallback
    return torch.device("cuda:0")
