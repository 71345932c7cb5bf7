"""Full-shape golden flushes: run the UNMODIFIED reference (HourunLi/LogKV) on CPU at G=8, D=128, K=12.

Test infrastructure only, beside ``make_golden.py`` (same import shim).  For every case of
``fullshape.py`` the reference cache is built at the production geometry, chunk 0 fills its
window, the pre-state is planted in the cluster buffers and in the host mirrors the reference
treats as authoritative (``_semantic_alive``, ``_semantic_p_hi_c``, ``_semantic_n_total``,
``_semantic_level0_phase``), ``begin_op_log()`` binds the route log, and chunks 1..3 are
committed with ``add_recent(..., record_op_log=True)`` (one 2048-token flush each).  After every
flush it records the decisions and layout fields in full (level counts, w, p_lo, p_hi, sum_wp,
order, pad, the cluster table, the exact pool's positions and spans, the op-log of per-token
cluster decisions) and, for the level K/V rows and the exact pool rows, per-(lane, level) bit
hashes plus float64 projections (``fullshape.bit_hash`` / ``projections``), which keeps the
fixture small.  It also times each flush (``add_recent`` wall time with the stated thread count).

Usage:  python tests/golden/make_fullshape.py --reference <checkout> [--out tests/golden] [--only NAME]
"""
from __future__ import annotations

import argparse
import json
import os
import sys
import time

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, HERE)
from fullshape import CASES, UNIFIED_CASES, bit_hash, make_case, prestate, projections  # noqa: E402
from make_golden import install_shim, to_np  # noqa: E402

THREADS = 8


def kv_digest(out: dict, prefix: str, name: str, t: torch.Tensor) -> None:
    """Bit hashes and projections of a [B, G, ..., rows, D] K/V buffer."""
    bits = to_np(t)
    if bits.dtype == np.float32:
        vals, bits = bits, bits.view(np.uint32)
    else:
        vals = t.float().numpy()
    out[f"{prefix}/{name}_hash"] = bit_hash(bits)
    out[f"{prefix}/{name}_proj"] = projections(vals)


def run_case(cfg: dict, outdir: str) -> tuple[str, list]:
    from litgpt.log_kv_cache import LogStructuredKVCache

    torch.set_num_threads(THREADS)
    inputs = make_case(cfg)
    dtype = torch.float32 if cfg["dtype"] == "fp32" else torch.bfloat16
    B, G, D = cfg["batch"], cfg["groups"], cfg["dim"]
    cache = LogStructuredKVCache(
        (B, G, cfg["max_seq"], D), (B, G, cfg["max_seq"], D), B=cfg["slots"], recent_size=cfg["recent"],
        dtype=dtype, semantic_clusters=True, cluster_k_max=cfg["clusters"], semantic_anchor_mode="mid",
        semantic_flush_granularity=cfg["granularity"], semantic_centroid_backend="sequential",
        semantic_replay_updates=True, allocate_second_order=False, alpha_exact_tokens=cfg["exact"],
        alpha_span_max_tokens=cfg["span_cap"], beta_novelty=cfg["beta"], beta_adaptive_merge=cfg["beta"],
        semantic_s_h=cfg["s_h"], cos_cache=torch.from_numpy(inputs["cos"]),
        sin_cache=torch.from_numpy(inputs["sin"]), rope_n_elem=D,
        semantic_unified_route=cfg.get("unified", False), semantic_merge_passes=cfg.get("merge_passes", 1))

    def push(chunk, record):
        k = torch.from_numpy(chunk["k"]).to(dtype)
        kr = torch.from_numpy(chunk["k_raw"]).to(dtype)
        v = torch.from_numpy(chunk["v"]).to(dtype)
        cache.add_recent(k, v, k_raw=kr, input_pos=torch.from_numpy(chunk["pos"]),
                         span_ends=chunk["span_ends"].tolist(), record_op_log=record)

    push(inputs["chunks"][0], False)
    pre = prestate(cfg, inputs)
    with torch.no_grad():
        for name, value in pre.items():
            getattr(cache, name).copy_(torch.from_numpy(value))
    cache._semantic_alive = pre["alive"].tolist()
    cache._semantic_p_hi_c = pre["p_hi_c"].astype(np.int64).tolist()
    cache._semantic_n_total = pre["n_total"].astype(np.int64).tolist()
    cache._semantic_level0_phase = pre["level0_phase"].astype(np.int64).tolist()
    cache.begin_op_log()
    out: dict = {}
    times = []
    for step in range(1, cfg["chunks"]):
        t0 = time.perf_counter()
        push(inputs["chunks"][step], True)
        times.append(time.perf_counter() - t0)
        p = f"flush{step}"
        for name in ("level_count", "level_w", "level_p_lo", "level_p_hi", "level_sum_wp", "level_order",
                     "pad_mask", "alive", "n_total", "p_hi_c", "level0_phase", "n_eff", "centroid", "alpha_pos",
                     "alpha_valid", "recent_pos"):
            out[f"{p}/{name}"] = to_np(getattr(cache, name))
        for name in ("level_k", "level_v", "alpha_k_raw", "alpha_v", "recent_k_raw", "recent_v"):
            kv_digest(out, p, name, getattr(cache, name))
        spans = cache._alpha_spans
        width = max(len(r) for r in spans)
        table = np.zeros((B, max(width, 1), 2), dtype=np.int64)
        for b, row in enumerate(spans):
            for i, (length, closed) in enumerate(row):
                table[b, i] = (length, int(closed))
        out[f"{p}/alpha_spans"] = table
        out[f"{p}/alpha_nspans"] = np.asarray([len(r) for r in spans], dtype=np.int64)
        out[f"{p}/scalars"] = np.asarray([cache.alpha_count, cache.recent_count, cache.token_count,
                                          cache.B_prime, cache.L_alloc], dtype=np.int64)
        log, lengths = cache.take_op_log()
        out[f"{p}/op_log_len"] = to_np(lengths)
        if step == cfg["chunks"] - 1:
            out["op_log"] = to_np(log)
    path = os.path.join(outdir, f"fullshape_{cfg['name']}.npz")
    np.savez_compressed(path, **out)
    return path, times


def main() -> None:
    parser = argparse.ArgumentParser()
    parser.add_argument("--reference", default=os.environ.get("LOGKV_REFERENCE"))
    parser.add_argument("--out", default=HERE)
    parser.add_argument("--only", default=None)
    args = parser.parse_args()
    if not args.reference:
        raise SystemExit("pass --reference <reference checkout> or set LOGKV_REFERENCE")
    install_shim(args.reference)
    timing_path = os.path.join(args.out, "fullshape_timing.json")
    timing = json.load(open(timing_path)) if os.path.exists(timing_path) else {}
    for cfg in CASES + UNIFIED_CASES:
        if args.only and cfg["name"] != args.only:
            continue
        path, times = run_case(cfg, args.out)
        timing[cfg["name"]] = dict(flush_s=[round(t, 4) for t in times], threads=THREADS)
        print("wrote", path, os.path.getsize(path), "flush s:", [round(t, 3) for t in times], flush=True)
    with open(timing_path, "w") as fh:
        json.dump(timing, fh, indent=1, sort_keys=True)


if __name__ == "__main__":
    main()
