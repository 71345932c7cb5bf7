"""Device flush against the reference at the production shape, with the near-tie log.

Each case of ``tests/golden/fullshape.py`` (G=8, D=128, K=12, B'=125, three 2048-token flushes,
fp32 / bf16, s_h = 1 / 12 / 32, farthest-point seeding; and the unified route with s_h = 1 / 32 and
frozen-centre sweeps) runs through ``add_recent`` with the op-log
bound, and after every flush the cache is compared with the fixture the unmodified reference wrote
(``tests/golden/make_fullshape.py``): per-token cluster decisions (op-log rows), the exact pool,
every layout field, the cluster table and the level / pool K-V bits.  Decisions may differ only
where the flush's near-tie log (relative gap < 1e-6 between the two best candidates, or between a
value and its threshold) names that decision; every logged tie is printed with both candidates.
"""
from __future__ import annotations

import os
import sys

import numpy as np
import pytest
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(HERE, "golden"))
from fullshape import CASES, UNIFIED_CASES, case, make_case, prestate  # noqa: E402
from fullshape_check import CLUSTER, LAYOUT, Checker  # noqa: E402

pytestmark = pytest.mark.gpu


def build_cache(cfg, inputs):
    from logkv_b200.cache import LogStructuredKVCache
    dt = torch.float32 if cfg["dtype"] == "fp32" else torch.bfloat16
    shape = (cfg["batch"], cfg["groups"], cfg["max_seq"], cfg["dim"])
    return LogStructuredKVCache(
        shape, shape, B=cfg["slots"], recent_size=cfg["recent"], device="cuda", dtype=dt, semantic_clusters=True,
        cluster_k_max=cfg["clusters"], semantic_flush_granularity=cfg["granularity"], semantic_anchor_mode="mid",
        semantic_centroid_backend="sequential", semantic_replay_updates=True, allocate_second_order=False,
        alpha_exact_tokens=cfg["exact"], alpha_span_max_tokens=cfg["span_cap"], beta_novelty=cfg["beta"],
        beta_adaptive_merge=cfg["beta"], semantic_s_h=cfg["s_h"], cos_cache=torch.from_numpy(inputs["cos"]),
        sin_cache=torch.from_numpy(inputs["sin"]), rope_n_elem=cfg["dim"],
        semantic_unified_route=cfg.get("unified", False), semantic_merge_passes=cfg.get("merge_passes", 1))


def push(cache, chunk, record):
    dt = cache.level_k.dtype
    cache.add_recent(torch.from_numpy(chunk["k"]).to("cuda", dt), torch.from_numpy(chunk["v"]).to("cuda", dt),
                     k_raw=torch.from_numpy(chunk["k_raw"]).to("cuda", dt),
                     input_pos=torch.from_numpy(chunk["pos"]).cuda(), span_ends=chunk["span_ends"].tolist(),
                     record_op_log=record)


def bits_and_values(t: torch.Tensor):
    t = t.detach().cpu()
    if t.dtype == torch.bfloat16:
        return t.view(torch.int16).numpy().view(np.uint16), t.float().numpy()
    v = t.numpy()
    return v.view(np.uint32), v


@pytest.mark.parametrize("name", [c["name"] for c in CASES + UNIFIED_CASES])
def test_fullshape_flush_matches_reference(name, cascade_path):
    cfg = case(name)
    inputs = make_case(cfg)
    cache = build_cache(cfg, inputs)
    assert (cache.B_prime, cache.L_alloc) == (125, 7)
    push(cache, inputs["chunks"][0], False)
    with torch.no_grad():
        for field, value in prestate(cfg, inputs).items():
            getattr(cache, field).copy_(torch.from_numpy(value))
    cache.begin_op_log()
    cache.read_ties(clear=True)
    check = Checker(name, cfg["dtype"])
    prev = np.zeros((cfg["batch"], cfg["groups"]), dtype=np.int32)
    for step in range(1, cfg["chunks"]):
        push(cache, inputs["chunks"][step], True)
        torch.cuda.synchronize()
        assert cache.read_status() == 0
        ties = cache.read_ties(clear=True)
        assert cache.ties_dropped == 0
        for t in ties:
            print(f"{name} flush {step}: near tie {t}")
        log, lengths = cache.take_op_log()
        state = {f: getattr(cache, f).cpu().numpy() for f in LAYOUT + CLUSTER + ("alpha_pos", "alpha_valid")}
        bits, values = {}, {}
        for f in ("level_k", "level_v", "alpha_k_raw", "alpha_v", "recent_k_raw", "recent_v"):
            bits[f], values[f] = bits_and_values(getattr(cache, f))
        full = np.zeros((cfg["batch"], cfg["groups"], 3 * cfg["max_seq"], 4), np.int32)
        got_log = log.cpu().numpy()
        full[:, :, :got_log.shape[2]] = got_log
        check.check_flush(step, state, full, prev, lengths.cpu().numpy(), ties, bits, values)
        prev = lengths.cpu().numpy()
    print(f"{name}: waivers: {check.report()}")
