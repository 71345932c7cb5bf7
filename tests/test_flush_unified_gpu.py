"""Device unified (Ward / radius) route against the reference's unified streams.

The CUDA flush with ``semantic_unified_route=True`` must leave every buffer and host mirror equal
to the unmodified reference's after every ``add_recent`` of the seeded unified streams
(tests/golden/make_golden.py, ``UNIFIED_CONFIGS``): candidate passes with radius limits, global
passes with and without frozen-centre sweeps, Ward merges of old clusters' ladders, new clusters
in freed slots, exact-difference and Gram pair matrices; fp32 and bf16, with and without Beta.
"""
from __future__ import annotations

import numpy as np
import pytest
import torch

from fixtures import as_values, load
from streams import UNIFIED_CONFIGS, make_stream
from test_flush_gpu import FIELDS, host_values, push_chunk, torch_dtype

pytestmark = pytest.mark.gpu


def unified_config(name: str) -> dict:
    return next(c for c in UNIFIED_CONFIGS if c["name"] == name)


def make_unified_cache(cfg, stream):
    from logkv_b200.cache import LogStructuredKVCache
    dt = torch_dtype(cfg)
    cos, sin = torch.from_numpy(stream["cos"]), torch.from_numpy(stream["sin"])
    return LogStructuredKVCache(
        (cfg["batch"], cfg["groups"], cfg["max_seq"], cfg["dim"]), (cfg["batch"], cfg["groups"], cfg["max_seq"], cfg["dim"]),
        B=cfg["slots"], recent_size=cfg["recent"], device="cuda", dtype=dt, semantic_clusters=True,
        cluster_k_max=cfg["clusters"], semantic_anchor_mode="mid", semantic_flush_granularity=cfg["granularity"],
        semantic_centroid_backend="sequential", semantic_replay_updates=True, allocate_second_order=False,
        alpha_exact_tokens=cfg["exact"], alpha_span_max_tokens=cfg["span_cap"], beta_novelty=cfg["beta"],
        beta_adaptive_merge=cfg["beta"], semantic_s_h=cfg.get("s_h"), cos_cache=cos, sin_cache=sin,
        rope_n_elem=cfg["dim"], semantic_unified_route=True, semantic_merge_passes=cfg.get("merge_passes", 1))


@pytest.mark.parametrize("name", [c["name"] for c in UNIFIED_CONFIGS])
def test_device_unified_flush_matches_reference_stream(name):
    cfg = unified_config(name)
    stream = make_stream(cfg)
    ref_steps = load(name)
    cache = make_unified_cache(cfg, stream)
    assert (cache.B_prime, cache.L_alloc) == tuple(ref_steps[0]["scalars"][3:5])
    for step, (chunk, ref) in enumerate(zip(stream["chunks"], ref_steps)):
        push_chunk(cache, cfg, chunk)
        assert cache.read_status() == 0, step
        for field in FIELDS:
            if field not in ref:
                continue
            want = as_values(ref[field], field)
            got = host_values(getattr(cache, field))
            np.testing.assert_array_equal(got.astype(want.dtype), want, err_msg=f"step {step} {field}")
        assert [cache.alpha_count, cache.recent_count, cache.token_count] == ref["scalars"].tolist()[:3]
        for mirror in ("_semantic_counts", "_semantic_alive", "_semantic_p_hi_c", "_semantic_n_total",
                       "_semantic_level0_phase"):
            np.testing.assert_array_equal(np.asarray(getattr(cache, mirror), dtype=np.int64), ref[mirror],
                                          err_msg=f"step {step} {mirror}")


def test_unified_route_rejects_what_it_does_not_build():
    cfg = unified_config("fp32_unified")
    stream = make_stream(cfg)
    cache = make_unified_cache(cfg, stream)
    chunk = stream["chunks"][0]
    k = torch.from_numpy(chunk["k"]).to("cuda", torch_dtype(cfg))
    with pytest.raises(NotImplementedError):
        cache.add_recent(k, k, k_raw=k, record_op_log=True, span_ends=chunk["span_ends"].tolist())
