import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
for p in (ROOT, os.path.join(ROOT, "squirrel-rs_b200")):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a)")


def has_gpu():
    try:
        import torch
        return torch.cuda.is_available()
    except Exception:
        return False


@pytest.fixture(scope="session")
def gpu_lib():
    """The CUDA C-ABI library. On a GPU box a missing or unloadable build is an error,
    never a skip: there is no CPU fallback."""
    if not has_gpu():
        pytest.skip("no CUDA device")
    from sqb200 import lib as sqlib
    return sqlib.load()
