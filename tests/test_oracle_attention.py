"""Pin the attention oracle (plan, pack, slot attention) against the reference's own outputs.

CPU only.  For every attend step of every golden stream the fixture holds the
reference cache's state after the previous ``add_recent`` plus, for the chunk
about to be committed, the reference's mid-anchor plan, its torch packer's
output and its CPU slot-attention outputs (whole chunk and a two-token decode).
The oracle rebuilds plan and pack from that state and must match them exactly
(the mass coordinate within one unit in the last place of the storage dtype:
it is a float32 ``log``); its float64 attention must match the reference's
within the stated tolerance (2e-2 absolute for bf16, 1e-4 for fp32).
"""
from __future__ import annotations

import numpy as np
import pytest

from fixtures import CONFIGS, as_values, config, load, make_stream
from oracle import attention as A
from oracle.numerics import to_storage

TOL = {"bf16": 2e-2, "fp32": 1e-4}


def attend_cases():
    for cfg in CONFIGS:
        stream = make_stream(cfg)
        for step, chunk in enumerate(stream["chunks"]):
            if chunk["attend"] and step > 0:
                yield cfg["name"], step


CASES = list(attend_cases())


def build_inputs(name: str, step: int):
    cfg = config(name)
    stream = make_stream(cfg)
    steps = load(name)
    prev, ref = steps[step - 1], steps[step]
    chunk = stream["chunks"][step]
    dt = cfg["dtype"]
    st = {k: as_values(v, k) for k, v in prev.items()}
    rope_dt = cfg.get("rope_dtype", "fp32")
    cos, sin = stream["cos"], stream["sin"]
    if rope_dt == "bf16":
        cos, sin = to_storage(cos, "bf16"), to_storage(sin, "bf16")
    alpha_count, recent_count = int(prev["scalars"][0]), int(prev["scalars"][1])
    q = to_storage(chunk["q"], dt)
    k = to_storage(chunk["k"], dt)
    v = to_storage(chunk["v"], dt)
    return cfg, st, ref, dict(q=q, k=k, v=v, cos=cos, sin=sin, rope_dt=rope_dt, alpha_count=alpha_count,
                              recent_count=recent_count)


def pack(cfg, st, x, plan, T):
    dim = ((cfg["dim"] + 1 + 7) // 8) * 8
    return A.pack_mid(st["level_k"], st["level_v"], st["level_w"], plan, st["alpha_k_raw"], st["alpha_v"],
                      st["alpha_pos"], st["alpha_valid"], x["alpha_count"], st["recent_k"], st["recent_v"],
                      x["recent_count"], x["k"][:, :, :T], x["v"][:, :, :T], x["cos"], x["sin"], cfg["dim"],
                      dim, cfg["dtype"], x["rope_dt"])


@pytest.mark.parametrize("name,step", CASES)
def test_plan_matches_reference(name, step):
    cfg, st, ref, x = build_inputs(name, step)
    idx, anchors, valid = A.mid_plan(st["level_count"], st["level_w"], st["level_sum_wp"])
    np.testing.assert_array_equal(idx, ref["plan_idx"])
    np.testing.assert_array_equal(anchors, ref["plan_anchor"])
    np.testing.assert_array_equal(valid, ref["plan_valid"])


@pytest.mark.parametrize("name,step", CASES)
def test_pack_matches_reference(name, step):
    cfg, st, ref, x = build_inputs(name, step)
    plan = A.mid_plan(st["level_count"], st["level_w"], st["level_sum_wp"])
    ka, va = pack(cfg, st, x, plan, x["k"].shape[2])
    want_k, want_v = as_values(ref["pack_k"], "pack_k"), as_values(ref["pack_v"], "pack_v")
    assert ka.shape == want_k.shape and va.shape == want_v.shape
    kd = cfg["dim"]
    np.testing.assert_array_equal(va, want_v)
    np.testing.assert_array_equal(np.delete(ka, kd, axis=-1), np.delete(want_k, kd, axis=-1))
    ulp = np.spacing(np.abs(want_k[..., kd]).astype(np.float32)) * (65536 if cfg["dtype"] == "bf16" else 1)
    assert np.all(np.abs(ka[..., kd] - want_k[..., kd]) <= ulp)


@pytest.mark.parametrize("name,step", CASES)
@pytest.mark.parametrize("tokens", ["chunk", "decode"])
def test_slot_attention_matches_reference(name, step, tokens):
    cfg, st, ref, x = build_inputs(name, step)
    plan = A.mid_plan(st["level_count"], st["level_w"], st["level_sum_wp"])
    T = x["k"].shape[2] if tokens == "chunk" else 2
    ka, va = pack(cfg, st, x, plan, T)
    out = A.slot_attention(x["q"][:, :, :T], ka, va, cfg["dim"] ** -0.5, T, cfg["dim"], cfg["dtype"])
    want = ref["attention" if tokens == "chunk" else "decode_attention"].astype(np.float64)
    assert out.shape == want.shape
    err = np.abs(out - want).max()
    assert err <= TOL[cfg["dtype"]], err
