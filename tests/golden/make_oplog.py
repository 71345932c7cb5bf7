"""Golden op-logs: run the UNMODIFIED reference (HourunLi/LogKV) on CPU with op-log recording.

Test infrastructure only, beside ``make_golden.py`` (same streams, same import shim).  The
reference cache is built as there, ``begin_op_log()`` binds its per-(batch, group) route log
(``log_kv_cache.py:2006-2028``), every ``add_recent`` runs with ``record_op_log=True``, and after
every step ``take_op_log()`` (``:2030-2038``) gives the log rows [B, G, n, 4] (op, cluster,
argument, position) and the per-lane lengths; both are saved per step, with the step's
``level_count`` as a check that recording did not change the flush.

Usage:  python tests/golden/make_oplog.py --reference <checkout> [--out tests/golden] [--only NAME]
"""
from __future__ import annotations

import argparse
import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, HERE)
from make_golden import install_shim, to_np  # noqa: E402
from streams import CONFIGS, UNIFIED_CONFIGS, make_stream  # noqa: E402


def run_config(cfg: dict, outdir: str) -> str:
    from litgpt.log_kv_cache import LogStructuredKVCache

    torch.set_num_threads(4)
    stream = make_stream(cfg)
    dtype = torch.float32 if cfg["dtype"] == "fp32" else torch.bfloat16
    cos = torch.from_numpy(stream["cos"])
    sin = torch.from_numpy(stream["sin"])
    if cfg.get("rope_dtype", "fp32") == "bf16":
        cos, sin = cos.to(torch.bfloat16), sin.to(torch.bfloat16)
    cache = LogStructuredKVCache(
        (cfg["batch"], cfg["groups"], cfg["max_seq"], cfg["dim"]),
        (cfg["batch"], cfg["groups"], cfg["max_seq"], cfg["dim"]),
        B=cfg["slots"], recent_size=cfg["recent"], dtype=dtype,
        semantic_clusters=True, cluster_k_max=cfg["clusters"], semantic_anchor_mode="mid",
        semantic_flush_granularity=cfg["granularity"], semantic_centroid_backend="sequential",
        semantic_replay_updates=True, allocate_second_order=False,
        alpha_exact_tokens=cfg["exact"], alpha_span_max_tokens=cfg["span_cap"],
        beta_novelty=cfg["beta"], beta_adaptive_merge=cfg["beta"],
        semantic_s_h=cfg.get("s_h"), cos_cache=cos, sin_cache=sin, rope_n_elem=cfg["dim"],
        semantic_unified_route=cfg.get("unified", False), semantic_merge_passes=cfg.get("merge_passes", 1),
    )
    cache.begin_op_log()
    out: dict = {}
    for step, chunk in enumerate(stream["chunks"]):
        k = torch.from_numpy(chunk["k"]).to(dtype)
        kr = torch.from_numpy(chunk["k_raw"]).to(dtype)
        v = torch.from_numpy(chunk["v"]).to(dtype)
        pos = torch.from_numpy(chunk["pos"]) if chunk.get("pos") is not None else None
        cache.add_recent(k, v, k_raw=kr, input_pos=pos, span_ends=chunk["span_ends"].tolist(), record_op_log=True)
        log, lengths = cache.take_op_log()
        out[f"step{step}/op_log"] = to_np(log)
        out[f"step{step}/op_log_len"] = to_np(lengths)
        out[f"step{step}/level_count"] = to_np(cache.level_count)
    path = os.path.join(outdir, f"oplog_{cfg['name']}.npz")
    np.savez_compressed(path, **out)
    return path


def main() -> None:
    parser = argparse.ArgumentParser()
    parser.add_argument("--reference", default=os.environ.get("LOGKV_REFERENCE"))
    parser.add_argument("--out", default=HERE)
    parser.add_argument("--only", default=None)
    args = parser.parse_args()
    if not args.reference:
        raise SystemExit("pass --reference <reference checkout> or set LOGKV_REFERENCE")
    install_shim(args.reference)
    for cfg in CONFIGS + UNIFIED_CONFIGS:
        if args.only and cfg["name"] != args.only:
            continue
        path = run_config(cfg, args.out)
        print("wrote", path, os.path.getsize(path))


if __name__ == "__main__":
    main()
