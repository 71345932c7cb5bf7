"""Device read side (plan, pack, slot attention) against the reference's records and the oracle.

Each golden stream is replayed through the B200 cache (whose flush is bit-exact
with the reference); before every recorded attend step the cache's plan and
packed K/V must equal the reference's bit for bit (the mass coordinate, a
float32 ``log``, within one unit in the last place of the storage dtype), and
its slot attention over the whole chunk and over a two-token decode must match
the reference's output within 2e-2 absolute for bf16 and 1e-4 for fp32, and the
float64 oracle within the same bound.
"""
from __future__ import annotations

import numpy as np
import pytest
import torch

from fixtures import CONFIGS, as_values, config, load, make_stream
from oracle import attention as A
from oracle.numerics import to_storage
from test_flush_gpu import host_values, make_cache, push_chunk, torch_dtype

pytestmark = pytest.mark.gpu

TOL = {"bf16": 2e-2, "fp32": 1e-4}


def oracle_attention(cfg, stream, cache, chunk, T):
    """Oracle slot attention from the device cache's own state (copied to the host)."""
    dt = cfg["dtype"]
    st = {name: host_values(getattr(cache, name)) for name in
          ("level_k", "level_v", "level_w", "level_count", "level_sum_wp", "alpha_k_raw", "alpha_v", "alpha_pos",
           "alpha_valid", "recent_k", "recent_v")}
    cos, sin = stream["cos"], stream["sin"]
    rope_dt = cfg.get("rope_dtype", "fp32")
    if rope_dt == "bf16":
        cos, sin = to_storage(cos, "bf16"), to_storage(sin, "bf16")
    plan = A.mid_plan(st["level_count"], st["level_w"], st["level_sum_wp"])
    k = to_storage(chunk["k"][:, :, :T], dt)
    v = to_storage(chunk["v"][:, :, :T], dt)
    q = to_storage(chunk["q"][:, :, :T], dt)
    ka, va = A.pack_mid(st["level_k"], st["level_v"], st["level_w"], plan, st["alpha_k_raw"], st["alpha_v"],
                        st["alpha_pos"], st["alpha_valid"], cache.alpha_count, st["recent_k"], st["recent_v"],
                        cache.recent_count, k, v, cos, sin, cfg["dim"], ((cfg["dim"] + 8) // 8) * 8, dt, rope_dt)
    return A.slot_attention(q, ka, va, cfg["dim"] ** -0.5, T, cfg["dim"], dt)


@pytest.mark.parametrize("name", [c["name"] for c in CONFIGS])
def test_read_side_matches_reference(name):
    from logkv_b200 import log_kv_chunk_attention, pack_mid_kv
    cfg = config(name)
    stream = make_stream(cfg)
    ref_steps = load(name)
    cache = make_cache(cfg, stream)
    dt = torch_dtype(cfg)
    scale = cfg["dim"] ** -0.5
    pack_dim = ((cfg["dim"] + 1 + 7) // 8) * 8
    checked = 0
    for step, (chunk, ref) in enumerate(zip(stream["chunks"], ref_steps)):
        if chunk["attend"]:
            q = torch.from_numpy(chunk["q"]).to("cuda", dt)
            k = torch.from_numpy(chunk["k"]).to("cuda", dt)
            v = torch.from_numpy(chunk["v"]).to("cuda", dt)
            with torch.no_grad():
                idx, anchors, ones, valid = cache._semantic_attention_plan()
                np.testing.assert_array_equal(idx.cpu().numpy(), ref["plan_idx"], err_msg=f"step {step}")
                np.testing.assert_array_equal(anchors.cpu().numpy(), ref["plan_anchor"], err_msg=f"step {step}")
                np.testing.assert_array_equal(valid.cpu().numpy(), ref["plan_valid"], err_msg=f"step {step}")
                assert bool((ones == 1).all())
                ka, va = pack_mid_kv(cache, (idx, anchors, ones, valid), k, v, pack_dim, backend="torch")
                want_k, want_v = as_values(ref["pack_k"], "pack_k"), as_values(ref["pack_v"], "pack_v")
                got_k, got_v = host_values(ka), host_values(va)
                kd = cfg["dim"]
                np.testing.assert_array_equal(got_v, want_v, err_msg=f"step {step} pack_v")
                np.testing.assert_array_equal(np.delete(got_k, kd, -1), np.delete(want_k, kd, -1),
                                              err_msg=f"step {step} pack_k")
                ulp = np.spacing(np.abs(want_k[..., kd]).astype(np.float32)) * (65536 if dt == torch.bfloat16 else 1)
                assert np.all(np.abs(got_k[..., kd] - want_k[..., kd]) <= ulp), step
                for T, key in ((k.size(2), "attention"), (2, "decode_attention")):
                    out = log_kv_chunk_attention(cache, q[:, :, :T], k[:, :, :T], v[:, :, :T], scale, 0.0)
                    got = host_values(out).astype(np.float64)
                    want = ref[key].astype(np.float64)
                    assert got.shape == want.shape
                    err_ref = np.abs(got - want).max()
                    err_oracle = np.abs(got - oracle_attention(cfg, stream, cache, chunk, T)).max()
                    assert err_ref <= TOL[cfg["dtype"]], (step, T, err_ref)
                    assert err_oracle <= TOL[cfg["dtype"]], (step, T, err_oracle)
            checked += 1
        push_chunk(cache, cfg, chunk)
    assert checked >= 4
    assert int(cache._read.status.item()) == 0


def test_decode_shapes_and_causal_tail():
    """Odd chunk lengths split into power-of-two query blocks; causal_tail=0 sees every new token."""
    from logkv_b200 import log_kv_chunk_attention
    cfg = config("bf16_beta")
    stream = make_stream(cfg)
    cache = make_cache(cfg, stream)
    for chunk in stream["chunks"][:5]:
        push_chunk(cache, cfg, chunk)
    chunk = stream["chunks"][5]
    dt = torch_dtype(cfg)
    scale = cfg["dim"] ** -0.5
    for T in (1, 3, 7):
        q = torch.from_numpy(chunk["q"][:, :, :T]).to("cuda", dt)
        k = torch.from_numpy(chunk["k"][:, :, :T]).to("cuda", dt)
        v = torch.from_numpy(chunk["v"][:, :, :T]).to("cuda", dt)
        with torch.no_grad():
            out = log_kv_chunk_attention(cache, q, k, v, scale, 0.0)
        want = oracle_attention(cfg, stream, cache, chunk, T)
        assert np.abs(host_values(out) - want).max() <= TOL["bf16"], T
    with torch.no_grad():
        q = torch.from_numpy(chunk["q"][:, :, :4]).to("cuda", dt)
        k = torch.from_numpy(chunk["k"][:, :, :4]).to("cuda", dt)
        v = torch.from_numpy(chunk["v"][:, :, :4]).to("cuda", dt)
        full = log_kv_chunk_attention(cache, q, k, v, scale, 0.0, causal_tail=0)
        causal = log_kv_chunk_attention(cache, q, k, v, scale, 0.0)
    # The last query token sees every new token either way; earlier ones differ.
    torch.testing.assert_close(full[:, :, 3], causal[:, :, 3], atol=0, rtol=0)
    assert (full[:, :, 0] - causal[:, :, 0]).abs().max() > 0
