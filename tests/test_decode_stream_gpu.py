"""Decoding as the reference's model runs it, against the CPU oracle.

``logkv_b200.decode.LogKVDecoder`` reproduces litgpt/model.py:1219-1247, :1330-1352: a token
with nothing pending attends over the frozen cache and itself and becomes pending; the next one
attends over the cache and [pending, itself] (causal_tail=0) and the pair is committed with
add_recent, flushing when the window overflows.  After a prefill of three chunks of a seeded
golden stream, 48 decode tokens run through the decoder; every step's output must match the
float64 oracle attention over the cache state and those new tokens (bf16 / fp32 tolerance of the
attention tests), and after every committed pair (the window overflows, so flushes happen) the
cache must equal an oracle cache fed the same pairs through its add_recent, bit for bit.
"""
from __future__ import annotations

import numpy as np
import pytest
import torch

from fixtures import config, make_stream
from oracle import attention as A
from oracle.cache import OracleCache
from oracle.numerics import to_storage
from test_attention_gpu import TOL
from test_flush_gpu import host_values, make_cache, push_chunk, torch_dtype

pytestmark = pytest.mark.gpu
STATE = ("level_k", "level_v", "level_w", "level_count", "centroid", "alpha_pos", "alpha_valid", "recent_k",
         "recent_k_raw", "recent_v", "recent_pos", "p_hi_c")


def oracle_step(cfg, stream, cache, q, k, v):
    """Float64 oracle output of one query token over the device cache's state plus the new keys."""
    dt = cfg["dtype"]
    st = {name: host_values(getattr(cache, name)) for name in
          ("level_k", "level_v", "level_w", "level_count", "level_sum_wp", "alpha_k_raw", "alpha_v", "alpha_pos",
           "alpha_valid", "recent_k", "recent_v")}
    plan = A.mid_plan(st["level_count"], st["level_w"], st["level_sum_wp"])
    n = k.shape[2]
    ka, va = A.pack_mid(st["level_k"], st["level_v"], st["level_w"], plan, st["alpha_k_raw"], st["alpha_v"],
                        st["alpha_pos"], st["alpha_valid"], cache.alpha_count, st["recent_k"], st["recent_v"],
                        cache.recent_count, k, v, stream["cos"], stream["sin"], cfg["dim"],
                        ((cfg["dim"] + 8) // 8) * 8, dt, "fp32")
    qq = np.repeat(q, n, axis=2)   # one query row per new key; causal tail only for a single key
    return A.slot_attention(qq, ka, va, cfg["dim"] ** -0.5, 1 if n == 1 else 0, cfg["dim"], dt)[:, :, :1]


@pytest.mark.parametrize("name", ["bf16_beta", "fp32_beta"])
def test_paired_decode_matches_oracle(name):
    from logkv_b200.decode import LogKVDecoder
    cfg = config(name)
    stream = make_stream(cfg)
    cache = make_cache(cfg, stream)
    oc = OracleCache(batch=cfg["batch"], groups=cfg["groups"], max_seq=cfg["max_seq"], dim=cfg["dim"],
                     B=cfg["slots"], recent=cfg["recent"], clusters=cfg["clusters"], granularity=cfg["granularity"],
                     exact=cfg["exact"], span_cap=cfg["span_cap"], beta=cfg["beta"], dtype=cfg["dtype"],
                     s_h=cfg.get("s_h"))
    for chunk in stream["chunks"][:3]:
        push_chunk(cache, cfg, chunk)
        oc.add_recent(chunk["k"], chunk["v"], chunk["k_raw"], chunk["positions"], chunk["span_ends"])
    dt = torch_dtype(cfg)
    rng = np.random.default_rng(31)
    B, G, D, H = cfg["batch"], cfg["groups"], cfg["dim"], 2 * cfg["groups"]
    dec = LogKVDecoder(cache, D ** -0.5)
    pos0 = int(stream["chunks"][2]["positions"][0, -1]) + 1
    pend = None
    commits = 0
    for t in range(48):
        q = to_storage(rng.standard_normal((B, H, 1, D)).astype(np.float32), cfg["dtype"])
        kr = to_storage(rng.standard_normal((B, G, 1, D)).astype(np.float32), cfg["dtype"])
        v = to_storage(rng.standard_normal((B, G, 1, D)).astype(np.float32), cfg["dtype"])
        k = kr.copy()
        ends = [[bool(rng.random() < 0.3)] for _ in range(B)]
        dev = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to("cuda", dt)  # noqa: E731
        kn = k if pend is None else np.concatenate([pend[0], k], axis=2)
        vn = v if pend is None else np.concatenate([pend[1], v], axis=2)
        want = oracle_step(cfg, stream, cache, q, kn, vn)
        with torch.no_grad():
            out = dec.step(dev(q), dev(k), dev(v), k_raw=dev(kr), input_pos=torch.tensor([pos0 + t]).cuda(),
                           span_ends=ends)
        torch.cuda.synchronize()
        err = np.abs(host_values(out) - want).max()
        assert err <= TOL[cfg["dtype"]], (t, err)
        if pend is None:
            pend = (k, v, kr, ends)
            continue
        pos = np.broadcast_to(np.asarray([pos0 + t - 1, pos0 + t], np.int64), (B, 2))
        oc.add_recent(np.concatenate([pend[0], k], 2), np.concatenate([pend[1], v], 2),
                      np.concatenate([pend[2], kr], 2), pos, np.asarray([a + b for a, b in zip(pend[3], ends)]))
        pend = None
        commits += 1
        assert cache.read_status() == 0
        state = oc.state()
        for field in STATE:
            np.testing.assert_array_equal(host_values(getattr(cache, field)).astype(state[field].dtype),
                                          state[field], err_msg=f"token {t} {field}")
        assert cache.recent_count == oc.recent_count
    assert commits == 24 and cache.read_counters()["flushes"] >= 3
