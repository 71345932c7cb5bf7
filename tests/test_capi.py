"""The C-ABI library loads on a CPU-only host and exports every symbol the header declares."""
from __future__ import annotations

import ctypes
import os
import re

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "logkv_b200.h")


def declared_symbols():
    text = open(HEADER).read()
    return sorted(set(re.findall(r"LOGKV_API\s+[\w\s\*]+?\b(logkv_\w+)\s*\(", text)))


@pytest.fixture(scope="module")
def lib():
    from logkv_b200 import build
    build.build()
    from logkv_b200 import _lib
    return _lib.lib()


def test_header_declares_entry_points():
    names = declared_symbols()
    assert "logkv_flush" in names and "logkv_flush_workspace_bytes" in names


def test_library_exports_every_declared_symbol(lib):
    for name in declared_symbols():
        assert hasattr(lib, name), name
        assert isinstance(getattr(lib, name), ctypes._CFuncPtr)


def test_workspace_size_and_argument_checks(lib):
    from logkv_b200 import _lib
    layout = _lib.Layout(1, 8, 128, 12, 7, 125, 4096, 256, 64, 1, 1, 1.0, 2048.0, 1.0)
    n = lib.logkv_flush_workspace_bytes(ctypes.byref(layout), 2048)
    assert n > 0
    bad = _lib.Layout(1, 8, 128, 64, 7, 125, 4096, 256, 64, 1, 1, 1.0, 2048.0, 1.0)  # K > 32
    assert lib.logkv_flush_workspace_bytes(ctypes.byref(bad), 2048) == 0
    # Invalid arguments are rejected before anything is launched (no device needed).
    state = _lib.State()
    assert lib.logkv_flush(ctypes.byref(bad), ctypes.byref(state), 2048, 4096, None, 0, None) == -1
    assert lib.logkv_flush(ctypes.byref(layout), None, 2048, 4096, None, 0, None) == -4
