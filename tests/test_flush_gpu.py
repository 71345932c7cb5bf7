"""Device flush parity: the CUDA path against the reference's golden streams and the oracle.

Every buffer and every host mirror of the B200 cache must equal the
reference's after every ``add_recent`` of the seeded streams (integer, layout
and K/V fields bit for bit; the oracle reproduces the same fixtures on CPU).
"""
from __future__ import annotations

import numpy as np
import pytest
import torch

from fixtures import CONFIGS, as_values, config, load, make_stream

pytestmark = pytest.mark.gpu

FIELDS = ["level_count", "alive", "p_hi_c", "n_total", "level0_phase", "level_p_lo", "level_p_hi",
          "level_sum_wp", "level_order", "pad_mask", "level_w", "alpha_pos", "alpha_valid", "recent_pos",
          "level_k", "level_v", "alpha_k_raw", "alpha_v", "recent_k", "recent_k_raw", "recent_v",
          "centroid", "n_eff", "level_imp", "current_segment", "ward_cost", "s_h"]


def torch_dtype(cfg):
    return torch.float32 if cfg["dtype"] == "fp32" else torch.bfloat16


def make_cache(cfg, stream):
    from logkv_b200.cache import LogStructuredKVCache
    dt = torch_dtype(cfg)
    cos, sin = torch.from_numpy(stream["cos"]), torch.from_numpy(stream["sin"])
    if cfg.get("rope_dtype", "fp32") == "bf16":
        cos, sin = cos.to(torch.bfloat16), sin.to(torch.bfloat16)
    return LogStructuredKVCache(
        (cfg["batch"], cfg["groups"], cfg["max_seq"], cfg["dim"]), (cfg["batch"], cfg["groups"], cfg["max_seq"], cfg["dim"]),
        B=cfg["slots"], recent_size=cfg["recent"], device="cuda", dtype=dt, semantic_clusters=True,
        cluster_k_max=cfg["clusters"], semantic_anchor_mode="mid", semantic_flush_granularity=cfg["granularity"],
        semantic_centroid_backend="sequential", semantic_replay_updates=True, allocate_second_order=False,
        alpha_exact_tokens=cfg["exact"], alpha_span_max_tokens=cfg["span_cap"], beta_novelty=cfg["beta"],
        beta_adaptive_merge=cfg["beta"], semantic_s_h=cfg.get("s_h"), cos_cache=cos, sin_cache=sin,
        rope_n_elem=cfg["dim"])


def host_values(t: torch.Tensor) -> np.ndarray:
    t = t.detach().cpu()
    if t.dtype == torch.bfloat16:
        return t.float().numpy()
    return t.numpy()


def push_chunk(cache, cfg, chunk):
    dt = torch_dtype(cfg)
    k = torch.from_numpy(chunk["k"]).to("cuda", dt)
    kr = torch.from_numpy(chunk["k_raw"]).to("cuda", dt)
    v = torch.from_numpy(chunk["v"]).to("cuda", dt)
    pos = torch.from_numpy(chunk["pos"]).cuda() if chunk.get("pos") is not None else None
    cache.add_recent(k, v, k_raw=kr, input_pos=pos, span_ends=chunk["span_ends"].tolist())


@pytest.mark.parametrize("name", [c["name"] for c in CONFIGS])
def test_device_flush_matches_reference_stream(name, cascade_path):
    cfg = config(name)
    stream = make_stream(cfg)
    ref_steps = load(name)
    cache = make_cache(cfg, stream)
    assert (cache.B_prime, cache.L_alloc) == tuple(ref_steps[0]["scalars"][3:5])
    names = [n for n, _ in cache.named_buffers()]
    assert set(FIELDS) - {"s_h"} <= set(names)
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
        for b in range(cfg["batch"]):
            n = int(ref["alpha_nspans"][b])
            want = [(int(a), bool(c)) for a, c in ref["alpha_spans"][b, :n]]
            assert cache._alpha_spans[b] == want, (step, b)
            width = len(cache._alpha_positions[b])
            assert ref["alpha_positions"][b, :width].tolist() == cache._alpha_positions[b]
        for mirror in ("_semantic_counts", "_semantic_alive", "_semantic_p_hi_c", "_semantic_n_total",
                       "_semantic_level0_phase"):
            np.testing.assert_array_equal(np.asarray(getattr(cache, mirror), dtype=np.int64), ref[mirror],
                                          err_msg=f"step {step} {mirror}")
