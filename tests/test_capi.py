"""The C-ABI library loads on a CPU-only host and exports every symbol the header declares."""
from __future__ import annotations

import ctypes
import os
import re

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADERS = [os.path.join(ROOT, "include", n) for n in sorted(os.listdir(os.path.join(ROOT, "include")))
           if n.endswith(".h")]


def declared_symbols():
    text = "".join(open(h).read() for h in HEADERS)
    return sorted(set(re.findall(r"LOGKV_\w*API\s+[\w\s\*]+?\b(logkv_\w+)\s*\(", text)))


@pytest.fixture(scope="module")
def lib():
    from logkv_b200 import build
    build.build()
    from logkv_b200 import _lib
    return _lib.lib()


def test_header_declares_entry_points():
    names = declared_symbols()
    assert "logkv_flush" in names and "logkv_flush_workspace_bytes" in names
    for name in ("logkv_attention_plan", "logkv_pack_prefix", "logkv_pack_mid", "logkv_attention",
                 "logkv_attention_workspace_bytes", "logkv_pair_distances", "logkv_mirror", "logkv_unified_init",
                 "logkv_unified_step"):
        assert name in names


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


def test_unified_layout_checks(lib):
    from logkv_b200 import _lib
    layout = _lib.Layout(1, 8, 128, 12, 7, 125, 4096, 256, 64, 1, 1, 1.0, 2048.0, 1.0, _lib.ROUTE_UNIFIED, 1)
    attach = _lib.Layout(1, 8, 128, 12, 7, 125, 4096, 256, 64, 1, 1, 1.0, 2048.0, 1.0)
    n = lib.logkv_flush_workspace_bytes(ctypes.byref(layout), 2048)
    # The unified workspace holds each lane's (P + F + K)^2 float32 distances.
    assert n > lib.logkv_flush_workspace_bytes(ctypes.byref(attach), 2048) + 8 * (256 + 2048 + 12) ** 2 * 4
    for bad in (_lib.Layout(1, 8, 128, 12, 7, 125, 4096, 256, 64, 1, 1, 1.0, 2048.0, 1.0, 2, 1),   # unknown route
                _lib.Layout(1, 8, 128, 12, 7, 125, 4096, 256, 64, 1, 1, 1.0, 2048.0, 1.0, 1, 0),   # passes < 1
                _lib.Layout(1, 8, 128, 12, 7, 125, 8192, 256, 64, 1, 1, 1.0, 2048.0, 1.0, 1, 1)):  # rows > 4096
        assert lib.logkv_flush_workspace_bytes(ctypes.byref(bad), 4096 if bad.recent_capacity == 8192 else 2048) == 0
    out = (ctypes.c_int32 * 16)()
    assert lib.logkv_read_unified(ctypes.byref(attach), 2048, None, out, 16, None) == -4


def test_attention_argument_checks(lib):
    from logkv_b200 import _lib
    layout = _lib.Layout(1, 8, 128, 12, 7, 125, 4096, 256, 64, 1, 1, 1.0, 2048.0, 1.0)
    # decode shapes need split partials; a bf16 chunk needs none beyond the header
    assert lib.logkv_attention_workspace_bytes(ctypes.byref(layout), 16, 1, 10756) > 256
    assert lib.logkv_attention_workspace_bytes(ctypes.byref(layout), 16, 2048, 10756) == 256
    assert lib.logkv_attention_workspace_bytes(ctypes.byref(layout), 12, 1, 10756) == 0   # heads % groups
    state, pre, args = _lib.State(), _lib.Prefix(), _lib.AttentionArgs()
    assert lib.logkv_attention(ctypes.byref(layout), ctypes.byref(state), ctypes.byref(pre), ctypes.byref(args),
                               None, 0, None) == -4
    plan = _lib.Plan()
    assert lib.logkv_attention_plan(ctypes.byref(layout), ctypes.byref(state), ctypes.byref(plan), None) == -4


def test_unified_argument_checks(lib):
    """Null pointers and out-of-range shapes are refused before anything is launched."""
    from logkv_b200.plugin import Unified, _lib_plugin
    plug = _lib_plugin()
    assert plug.logkv_pair_distances(None, None, 1, 4, None) == -4
    assert plug.logkv_mirror(None, 1, 4, None) == -4
    assert plug.logkv_unified_init(None, None) == -4
    assert plug.logkv_unified_step(ctypes.byref(Unified()), None) == -4
    fake = ctypes.c_void_p(64)
    u = Unified(*([fake] * 3 + [None] + [fake] * 7), 1, 4097, 8, 1)
    assert plug.logkv_unified_init(ctypes.byref(u), None) == -1
    u = Unified(*([fake] * 3 + [None] + [fake] * 7), 0, 16, 8, 1)
    assert plug.logkv_unified_step(ctypes.byref(u), None) == -1


def test_constructor_rejects_unknown_keywords():
    """The cache takes the reference's keywords only (litgpt/log_kv_cache.py:681-720): a misspelt
    YAML switch raises TypeError instead of being dropped; the reference's defaults (no semantic
    clusters, multi anchors) are outside this path and raise NotImplementedError."""
    from logkv_b200.cache import LogStructuredKVCache
    with pytest.raises(TypeError):
        LogStructuredKVCache((1, 1, 64, 8), (1, 1, 64, 8), semantic_clusterz=True)
    with pytest.raises(NotImplementedError):
        LogStructuredKVCache((1, 1, 64, 8), (1, 1, 64, 8), device="cpu")
