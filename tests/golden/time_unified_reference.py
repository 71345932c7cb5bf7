"""Time the UNMODIFIED reference's CPU unified route at the unified stress shape (test infrastructure).

BASELINE configs[4]'s per-stream shape: one stream, 8 KV groups, head dim 128, bf16 K/V, K = 12,
B = 128, recent window 2048 flushed 2048 tokens at a time, exact pool 256 (span cap 64), Beta on,
``semantic_unified_route=True``, keys from ``logkv_b200.workload.StressMixture`` (48 components,
sigma ~ U[0.1, 0.6], 10 % orphans).  Chunk 0 fills the window; chunks 1..3 each flush 2048 tokens
through ``add_recent``, whose wall time is recorded (torch CPU threads stated) in
``unified_timing.json`` beside this script.  Reads the reference checkout through the import shim
of ``make_golden.py``; it is never run where the checkout is absent.

Usage:  python tests/golden/time_unified_reference.py --reference <checkout> [--threads 8]
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
sys.path.insert(0, os.path.dirname(os.path.dirname(HERE)))
from make_golden import install_shim  # noqa: E402
from logkv_b200.workload import StressMixture, apply_rope, rope_tables  # noqa: E402

G, D, K, SLOTS, RECENT, EXACT, SPAN, MAX_SEQ, T = 8, 128, 12, 128, 2048, 256, 64, 65536, 2048


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default=os.environ.get("LOGKV_REFERENCE"))
    ap.add_argument("--threads", type=int, default=8)
    ap.add_argument("--flushes", type=int, default=3)
    args = ap.parse_args()
    install_shim(args.reference)
    from litgpt.log_kv_cache import LogStructuredKVCache
    torch.set_num_threads(args.threads)
    rng = np.random.default_rng(2024)
    keys = StressMixture(rng, 1, G, D)
    cos, sin = rope_tables(MAX_SEQ + 64, D)
    cache = LogStructuredKVCache(
        (1, G, MAX_SEQ, D), (1, G, MAX_SEQ, D), B=SLOTS, recent_size=RECENT, dtype=torch.bfloat16,
        semantic_clusters=True, cluster_k_max=K, semantic_anchor_mode="mid", semantic_flush_granularity=T,
        semantic_centroid_backend="sequential", allocate_second_order=False, alpha_exact_tokens=EXACT,
        alpha_span_max_tokens=SPAN, beta_novelty=True, beta_adaptive_merge=True, cos_cache=torch.from_numpy(cos),
        sin_cache=torch.from_numpy(sin), rope_n_elem=D, semantic_unified_route=True)
    times = []
    for c in range(args.flushes + 1):
        kr = keys.draw(T)
        pos = np.arange(c * T, (c + 1) * T)[None, :]
        k = apply_rope(kr, pos[:, None, :], cos, sin)
        v = rng.standard_normal((1, G, T, D)).astype(np.float32)
        ends = [(np.arange(T) % 23 == 22).tolist()]
        t0 = time.perf_counter()
        cache.add_recent(torch.from_numpy(k).bfloat16(), torch.from_numpy(v).bfloat16(),
                         k_raw=torch.from_numpy(kr).bfloat16(), span_ends=ends)
        if c:
            times.append(time.perf_counter() - t0)
        print("chunk", c, "s", round(time.perf_counter() - t0, 3), flush=True)
    out = dict(flush_s=[round(t, 3) for t in times], threads=args.threads, streams=1, groups=G, head_dim=D,
               tokens_per_flush=T, shape="BASELINE configs[4] per stream (bf16, K=12, B=128, recent 2048, exact 256)",
               route="reference CPU Torch path, semantic_unified_route=True (_UnifiedReduceTorch)")
    with open(os.path.join(HERE, "unified_timing.json"), "w") as fh:
        json.dump(out, fh, indent=1)
    print(out)


if __name__ == "__main__":
    main()
