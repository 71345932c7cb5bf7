"""The CPU oracle against the reference at the production shape (tests/golden/fullshape_*.npz).

The fixtures come from the unmodified reference (``tests/golden/make_fullshape.py``): one layer at
G=8, D=128, K=12, B'=125, three 2048-token flushes per case, fp32 and bf16, s_h = 1 / 12 / 32 and a
case with 4 of 12 clusters opened by farthest-point seeding.  The oracle keeps one canonical
summation order; at this shape it must still reproduce every decision and layout field, the
cluster table (centroids and n_eff bit for bit) and the level K/V bits of the reference.
"""
from __future__ import annotations

import os
import sys

import numpy as np
import pytest

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(HERE, "golden"))
from fullshape import CASES, bit_hash, case, make_case, prestate  # noqa: E402
from fullshape_check import CLUSTER, LAYOUT, load  # noqa: E402


@pytest.mark.parametrize("name", [c["name"] for c in CASES])
def test_oracle_matches_reference_at_full_shape(name):
    from oracle.cache import OracleCache
    cfg = case(name)
    inputs = make_case(cfg)
    ref = load(name)
    oc = OracleCache(batch=cfg["batch"], groups=cfg["groups"], max_seq=cfg["max_seq"], dim=cfg["dim"], B=cfg["slots"],
                     recent=cfg["recent"], clusters=cfg["clusters"], granularity=cfg["granularity"],
                     exact=cfg["exact"], span_cap=cfg["span_cap"], beta=cfg["beta"], dtype=cfg["dtype"],
                     s_h=cfg["s_h"])
    chunks = inputs["chunks"]
    c0 = chunks[0]
    oc.add_recent(c0["k"], c0["v"], c0["k_raw"], c0["pos"][None], c0["span_ends"])
    for field, value in prestate(cfg, inputs).items():
        getattr(oc, field)[...] = value
    for step in range(1, cfg["chunks"]):
        c = chunks[step]
        oc.add_recent(c["k"], c["v"], c["k_raw"], c["pos"][None], c["span_ends"])
        st, p = oc.state(), f"flush{step}"
        assert [oc.alpha_count, oc.recent_count, oc.token_count, oc.B_prime, oc.L] == ref[f"{p}/scalars"].tolist()
        for field in LAYOUT + CLUSTER + ("alpha_pos", "alpha_valid", "recent_pos"):
            want = ref[f"{p}/{field}"]
            np.testing.assert_array_equal(np.asarray(st[field]).astype(want.dtype), want, err_msg=f"flush {step} {field}")
        for field in ("level_k", "level_v", "alpha_k_raw", "alpha_v", "recent_k_raw", "recent_v"):
            vals = np.ascontiguousarray(st[field], dtype=np.float32)
            bits = vals.view(np.uint32) if cfg["dtype"] == "fp32" else (vals.view(np.uint32) >> 16).astype(np.uint16)
            np.testing.assert_array_equal(bit_hash(bits), ref[f"{p}/{field}_hash"], err_msg=f"flush {step} {field}")
        spans = [(int(a), bool(b)) for a, b in ref[f"{p}/alpha_spans"][0, :int(ref[f"{p}/alpha_nspans"][0])]]
        assert [(int(a), bool(b)) for a, b in oc.alpha_spans[0]] == spans


def test_checker_waives_only_logged_ties(monkeypatch):
    """A decision that differs from the reference passes only with a near-tie entry naming it."""
    import fullshape_check as fc
    ref = load("f32_sh12")
    chk = fc.Checker("f32_sh12", "fp32")
    # K/V hashes are compared elsewhere; here they always match.
    monkeypatch.setattr("fullshape.bit_hash", lambda bits: bits)
    bits = {f: ref[f"flush1/{f}_hash"] for f in ("level_k", "level_v", "alpha_k_raw", "alpha_v", "recent_k_raw",
                                                 "recent_v")}
    state = {f: ref[f"flush1/{f}"] for f in LAYOUT + CLUSTER + ("alpha_pos", "alpha_valid")}
    lengths = ref["flush1/op_log_len"]
    log = ref["op_log"].copy()
    # Plant a flipped decision on the CPU: lane (0, 3), first JOIN row of the flush.
    row = next(i for i in range(int(lengths[0, 3])) if log[0, 3, i, 0] == 2)
    log[0, 3, row, 1] = (log[0, 3, row, 1] + 1) % 12
    pos = int(log[0, 3, row, 3])
    zero = np.zeros_like(lengths)
    with pytest.raises(AssertionError, match="without a logged near tie"):
        chk.check_flush(1, state, log, zero, lengths, [], bits, {})
    chk = fc.Checker("f32_sh12", "fp32")
    tie = dict(kind="direct", batch=0, group=3, index=pos, first=1, second=0, gap=1e-7, value=12.0, flush=0,
               cluster=-1)
    chk.check_flush(1, state, log, zero, lengths, [tie], bits, {})
    assert chk.waivers and chk.waivers[0][1] == "decision" and (0, 3) in chk.waived_lanes
