"""The allocation-free flush entry point agrees with the workspace entry point.

``logkv_flush_static`` serves callers that may not allocate device memory
(hosts that lock their GPU allocator after start-up, bindings that cannot hand
a device buffer across the C ABI): it flushes through scratch compiled into the
library instead of a caller workspace.  Two caches receive the same seeded
stream; one flushes through ``logkv_flush`` (its own workspace), the other
through ``logkv_flush_static`` called directly via ctypes.  After each of two
consecutive static flushes every buffer must match bit for bit, the tolerance
all flush parity tests here use, and the region's status word (read with a NULL
workspace) must be clear.  A cache of another layout (float32, its own stream of
inputs) then flushes through the same region on the same stream, leaving its
data there, and the first cache's next static flush must still match.  This
file is collected last so that a run that stops at the first failure has run
every other test before it.
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
    cache._ladder_epoch += 1   # what LogStructuredKVCache.flush_device does before its own launch
    state = cache._state_struct()
    code = fn(ctypes.byref(cache._layout), ctypes.byref(state), int(take), int(cache.recent_count),
              ctypes.c_void_p(_lib.stream_ptr(cache.level_k.device)))
    _lib.check(code, "logkv_flush_static")


def static_status(device) -> int:
    """Status word of the last static flush on the current device (logkv_read_status with NULL)."""
    from logkv_b200 import _lib
    out = ctypes.c_int32(-1)
    _lib.check(_lib.lib().logkv_read_status(None, ctypes.byref(out), ctypes.c_void_p(_lib.stream_ptr(device))),
               "logkv_read_status")
    return int(out.value)


class Pair:
    """A workspace cache and a static-scratch cache fed the same stream."""

    def __init__(self, name: str):
        from test_flush_gpu import make_cache
        self.cfg = config(name)
        self.stream = make_stream(self.cfg)
        self.ref = make_cache(self.cfg, self.stream)
        self.static = make_cache(self.cfg, self.stream)
        self.static.flush_device = lambda take: static_flush(self.static, take)
        self.chunks = iter(self.stream["chunks"])

    def next_flush(self) -> None:
        """Push chunks until one flush happened in both caches, then compare them."""
        from test_flush_gpu import push_chunk
        while True:
            chunk = next(self.chunks)
            before = self.ref.read_counters()["flushes"]
            push_chunk(self.ref, self.cfg, chunk)
            push_chunk(self.static, self.cfg, chunk)
            torch.cuda.synchronize()
            if self.ref.read_counters()["flushes"] != before:
                break
        assert static_status(self.static.level_k.device) == 0
        assert self.ref.read_status() == 0
        for name in FIELDS:
            a, b = getattr(self.ref, name), getattr(self.static, name)
            assert torch.equal(a, b), f"{self.cfg['name']}: {name}"
        assert self.ref._alpha_spans == self.static._alpha_spans
        assert self.ref.alpha_count == self.static.alpha_count
        assert self.ref._ladder_epoch == self.static._ladder_epoch


def test_static_scratch_flush_matches_workspace_flush():
    main = Pair("bf16_beta")
    main.next_flush()
    main.next_flush()            # two static flushes in a row
    other = Pair("fp32_beta")    # another layout's data now sits in the shared region
    other.next_flush()
    main.next_flush()
    # Layouts needing more scratch than the fixed region are refused before any launch.
    from logkv_b200 import _lib
    big = _lib.Layout(1, 8, 128, 12, 7, 125, 4096, 256, 64, 1, 1, 1.0, 2048.0, 1.0)
    fn = _lib.lib().logkv_flush_static
    assert fn(ctypes.byref(big), ctypes.byref(main.ref._state_struct()), 2048, 4096, None) == -3
    np.testing.assert_equal(main.ref.read_status(), 0)
