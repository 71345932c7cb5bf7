"""Flushes of caches holding a single KV group (what one rank of an 8-way KV-head shard of an
8-group model holds) against the oracle, bit for bit, for the attach and the unified route."""
from __future__ import annotations

import numpy as np
import pytest

from fixtures import config
from streams import UNIFIED_CONFIGS, make_stream
from test_flush_gpu import host_values, make_cache, push_chunk
from test_flush_unified_gpu import make_unified_cache
from test_oracle_golden import oracle_for
from test_oracle_unified_stream import unified_oracle

pytestmark = pytest.mark.gpu

FIELDS = ("level_count", "level_k", "level_v", "level_w", "level_p_lo", "level_p_hi", "level_sum_wp", "level_order",
          "pad_mask", "centroid", "n_eff", "n_total", "p_hi_c", "alive", "alpha_pos", "alpha_valid", "alpha_k_raw",
          "recent_k_raw")


@pytest.mark.parametrize("name", ["fp32_beta", "bf16_beta", "fp32_unified", "bf16_unified_nobeta"])
def test_one_group_flush_matches_oracle(name):
    unified = "unified" in name
    cfg = dict(next(c for c in UNIFIED_CONFIGS if c["name"] == name) if unified else config(name), groups=1)
    stream = make_stream(cfg)
    cache = make_unified_cache(cfg, stream) if unified else make_cache(cfg, stream)
    oc = unified_oracle(cfg) if unified else oracle_for(cfg)
    for step, chunk in enumerate(stream["chunks"]):
        push_chunk(cache, cfg, chunk)
        oc.add_recent(chunk["k"], chunk["v"], chunk["k_raw"], chunk["positions"], chunk["span_ends"])
        assert cache.read_status() == 0, step
        ref = oc.state()
        for field in FIELDS:
            want = np.asarray(ref[field])
            got = host_values(getattr(cache, field)).astype(want.dtype)
            np.testing.assert_array_equal(got, want, err_msg=f"step {step} {field}")
