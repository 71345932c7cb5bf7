"""Pin the oracle's flush-level unified (Ward / radius) route against the reference itself.

CPU only.  The fixtures were produced by the unmodified reference cache with
``semantic_unified_route=True`` (tests/golden/make_golden.py, ``UNIFIED_CONFIGS``): candidate
passes with radius limits, global passes to K with and without frozen-centre sweeps
(``semantic_merge_passes``), Ward merges of old clusters' ladders, new clusters in freed
slots, fp32 and bf16, with and without Beta.  The oracle replays the same seeded streams and
must reproduce every buffer and host mirror after every ``add_recent``.
"""
from __future__ import annotations

import pytest

from fixtures import load
from streams import UNIFIED_CONFIGS, make_stream
from test_oracle_golden import compare_state
from oracle.cache import OracleCache


def unified_config(name: str) -> dict:
    return next(c for c in UNIFIED_CONFIGS if c["name"] == name)


def unified_oracle(cfg) -> OracleCache:
    return OracleCache(batch=cfg["batch"], groups=cfg["groups"], max_seq=cfg["max_seq"], dim=cfg["dim"],
                       B=cfg["slots"], recent=cfg["recent"], clusters=cfg["clusters"],
                       granularity=cfg["granularity"], exact=cfg["exact"], span_cap=cfg["span_cap"],
                       beta=cfg["beta"], dtype=cfg["dtype"], s_h=cfg.get("s_h"), unified=True,
                       merge_passes=cfg.get("merge_passes", 1))


@pytest.mark.parametrize("name", [c["name"] for c in UNIFIED_CONFIGS])
def test_oracle_replays_reference_unified_stream(name):
    cfg = unified_config(name)
    stream = make_stream(cfg)
    ref_steps = load(name)
    oc = unified_oracle(cfg)
    assert (oc.B_prime, oc.L) == tuple(ref_steps[0]["scalars"][3:5])
    ward = 0
    for step, (chunk, ref) in enumerate(zip(stream["chunks"], ref_steps)):
        oc.add_recent(chunk["k"], chunk["v"], chunk["k_raw"], chunk["positions"], chunk["span_ends"])
        compare_state(oc, ref, step)
        for flush in oc.trace:
            for d in flush.get("unified", {}).values():
                ward += int(len(d["gtrace"]) and (d["gtrace"][:, 1] < 0).sum() == 0)
