"""The allocation-free flush entry point agrees with the workspace entry point.

``logkv_flush_static`` serves callers that may not allocate device memory
(hosts that lock their GPU allocator after start-up, bindings that cannot hand
a device buffer across the C ABI): it flushes through scratch compiled into the
library instead of a caller workspace.  Two caches receive the same seeded
stream; one flushes through ``logkv_flush`` (its own workspace), the other
through ``logkv_flush_static`` called directly via ctypes.  After each of two
consecutive flushes every buffer must match bit for bit, the tolerance all
flush parity tests here use.  This file is collected last so that a run that
stops at the first failure has run every other test before it.
"""
from __future__ import annotations

import ctypes

import numpy as np
import pytest
import torch

from fixtures import config, make_stream

pytestmark = pytest.mark.gpu

FIELDS = ["level_k", "level_v", "level_w", "level_p_lo", "level_p_hi", "level_sum_wp", "level_order", "pad_mask",
          "level_count", "centroid", "n_eff", "n_total", "p_hi_c", "level0_phase", "alive", "recent_k",
          "recent_k_raw", "recent_v", "recent_pos", "alpha_k_raw", "alpha_v", "alpha_pos", "alpha_valid"]


def static_flush(cache, take: int) -> None:
    """Flush ``cache`` through logkv_flush_static (no workspace), via the C ABI."""
    from logkv_b200 import _lib
    fn = _lib.lib().logkv_flush_static
    fn.restype = ctypes.c_int
    fn.argtypes = [ctypes.POINTER(_lib.Layout), ctypes.POINTER(_lib.State), ctypes.c_int32, ctypes.c_int32,
                   ctypes.c_void_p]
    state = cache._state_struct()
    code = fn(ctypes.byref(cache._layout), ctypes.byref(state), int(take), int(cache.recent_count),
              ctypes.c_void_p(_lib.stream_ptr(cache.level_k.device)))
    _lib.check(code, "logkv_flush_static")


def test_static_scratch_flush_matches_workspace_flush():
    from test_flush_gpu import make_cache, push_chunk
    cfg = config("bf16_beta")
    stream = make_stream(cfg)
    ref = make_cache(cfg, stream)
    static = make_cache(cfg, stream)
    static.flush_device = lambda take: static_flush(static, take)
    flushes = 0
    for chunk in stream["chunks"]:
        before = ref.read_counters()["flushes"]
        push_chunk(ref, cfg, chunk)
        push_chunk(static, cfg, chunk)
        torch.cuda.synchronize()
        if ref.read_counters()["flushes"] == before:
            continue
        flushes += 1
        for name in FIELDS:
            a, b = getattr(ref, name), getattr(static, name)
            assert torch.equal(a, b), f"flush {flushes}: {name}"
        assert ref._alpha_spans == static._alpha_spans
        assert ref.alpha_count == static.alpha_count
        if flushes == 2:
            break
    assert flushes == 2
    # Layouts needing more scratch than the fixed region are refused before any launch.
    from logkv_b200 import _lib
    big = _lib.Layout(1, 8, 128, 12, 7, 125, 4096, 256, 64, 1, 1, 1.0, 2048.0, 1.0)
    fn = _lib.lib().logkv_flush_static
    assert fn(ctypes.byref(big), ctypes.byref(ref._state_struct()), 2048, 4096, None) == -3
    np.testing.assert_equal(ref.read_status(), 0)
