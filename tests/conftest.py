import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA B200 (sm_100a) device")


@pytest.fixture(params=["parallel", "sequential"])
def cascade_path(request, monkeypatch):
    """Run a flush test through both ladder cascades of the library: the parallel merge / move
    kernels (the default) and the sequential per-lane walk (LOGKV_CASCADE=sequential)."""
    if request.param == "sequential":
        monkeypatch.setenv("LOGKV_CASCADE", "sequential")
    else:
        monkeypatch.delenv("LOGKV_CASCADE", raising=False)
    return request.param
