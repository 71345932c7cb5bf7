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
    # Near ties of the Ward decisions (row minima, budget cuts) are logged, not waived: every
    # entry is a real one (gap below 1e-6, finite costs, a row of its pass, distinct columns).
    ties = [t for t in cache.read_ties() if t["kind"] in ("ward_min", "ward_budget")]
    for t in ties:
        print("ward near tie", t)
        assert t["gap"] < 1e-6 and np.isfinite(t["value"]) and t["cluster"] in (0, 1), t
        assert t["first"] != t["second"] and 0 <= t["index"] < cache.max_seq_length + cfg["clusters"], t


@pytest.mark.parametrize("name", [c["name"] for c in UNIFIED_CONFIGS])
def test_unified_op_log_matches_reference(name):
    """WARD_MERGE, NEW_CLUSTER and JOIN rows after every step equal the reference's op-log
    (tests/golden/oplog_<name>.npz from make_oplog.py), and recording leaves the flush unchanged."""
    import os
    cfg = unified_config(name)
    stream = make_stream(cfg)
    ref = np.load(os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", f"oplog_{name}.npz"))
    cache = make_unified_cache(cfg, stream)
    cache.begin_op_log()
    for step, chunk in enumerate(stream["chunks"]):
        dt = cache.level_k.dtype
        k = torch.from_numpy(chunk["k"]).to("cuda", dt)
        kr = torch.from_numpy(chunk["k_raw"]).to("cuda", dt)
        v = torch.from_numpy(chunk["v"]).to("cuda", dt)
        pos = torch.from_numpy(chunk["pos"]).cuda() if chunk.get("pos") is not None else None
        cache.add_recent(k, v, k_raw=kr, input_pos=pos, span_ends=chunk["span_ends"].tolist(), record_op_log=True)
        log, lengths = cache.take_op_log()
        want_len = ref[f"step{step}/op_log_len"]
        np.testing.assert_array_equal(lengths.cpu().numpy(), want_len, err_msg=f"step {step} lengths")
        want, got = ref[f"step{step}/op_log"], log.cpu().numpy()
        for b in range(want.shape[0]):
            for g in range(want.shape[1]):
                n = int(want_len[b, g])
                np.testing.assert_array_equal(got[b, g, :n], want[b, g, :n], err_msg=f"step {step} lane {(b, g)}")
        np.testing.assert_array_equal(cache.level_count.cpu().numpy(), ref[f"step{step}/level_count"])


@pytest.mark.parametrize("name", ["bf16_unified_nobeta", "fp32_unified_passes2", "fp32_unified_sh"])
def test_unified_update_tape_replays_without_routing(name):
    """Record every flush of a unified stream on an update tape (Ward merges and their Beta cuts
    included), reset the cache, and replay: no flush reroutes, and every buffer equals the recorded
    run after every step, twice."""
    from unittest.mock import patch
    from logkv_b200 import _SemanticReplayUpdates
    from test_update_tape_gpu import assert_state, state
    cfg = unified_config(name)
    stream = make_stream(cfg)
    cache = make_unified_cache(cfg, stream)
    tape = _SemanticReplayUpdates()
    expected = []
    dt = torch_dtype(cfg)

    def push(chunk, **kw):
        k = torch.from_numpy(chunk["k"]).to("cuda", dt)
        kr = torch.from_numpy(chunk["k_raw"]).to("cuda", dt)
        v = torch.from_numpy(chunk["v"]).to("cuda", dt)
        pos = torch.from_numpy(chunk["pos"]).cuda() if chunk.get("pos") is not None else None
        cache.add_recent(k, v, k_raw=kr, input_pos=pos, span_ends=chunk["span_ends"].tolist(), **kw)

    with torch.no_grad(), cache._semantic_update_context(tape):
        for chunk in stream["chunks"]:
            push(chunk, record_op_log=True)
            expected.append(state(cache))
    for _ in range(2):
        cache.reset_parameters()
        with patch.object(cache, "flush_device", side_effect=AssertionError("rerouted")):
            for chunk, want in zip(stream["chunks"], expected):
                with torch.no_grad(), cache._semantic_update_context(tape, replay=True):
                    push(chunk)
                assert cache.read_status() == 0
                assert_state(cache, want)


def test_unified_ward_ties_are_logged():
    """Duplicated tokens make exactly equal Ward costs: the row minima that they decide (by the
    XOR index rule, the same on both sides) are logged as WARD_MIN near ties, and the cache still
    equals the oracle's bit for bit after every step."""
    from test_oracle_unified_stream import unified_oracle
    cfg = unified_config("fp32_unified_sh")
    stream = make_stream(cfg)
    for chunk in stream["chunks"]:
        for key in ("k", "k_raw"):
            chunk[key][:, :, 1::7] = chunk[key][:, :, 0:-1:7][:, :, :chunk[key][:, :, 1::7].shape[2]]
    cache = make_unified_cache(cfg, stream)
    oc = unified_oracle(cfg)
    for step, chunk in enumerate(stream["chunks"][:8]):
        push_chunk(cache, cfg, chunk)
        oc.add_recent(chunk["k"], chunk["v"], chunk["k_raw"], chunk["positions"], chunk["span_ends"])
        assert cache.read_status() == 0, step
        ref = oc.state()
        for name in ("level_count", "level_k", "level_v", "level_w", "level_p_lo", "level_order", "centroid",
                     "n_eff", "n_total", "alive"):
            want = np.asarray(ref[name])
            got = host_values(getattr(cache, name)).astype(want.dtype)
            np.testing.assert_array_equal(got, want, err_msg=f"step {step} {name}")
    ties = [t for t in cache.read_ties() if t["kind"] == "ward_min"]
    assert ties, "duplicated tokens must leave logged Ward near ties"
    assert all(t["gap"] == 0.0 for t in ties[:50]) or all(t["gap"] < 1e-6 for t in ties)
