"""Small seeded streaming workloads shared by the golden generator and the tests.

Each config is a miniature of the flush-and-attend path (few groups, small
head dim, a handful of clusters) so the reference's CPU path and the oracle
finish in seconds, while every branch of the flush is still reached: cluster
seeding on the first flush, direct joins and orphans, Alpha span eviction
(late re-insertion into older clusters), Beta 4->2 cuts and multi-level
carries.
"""
from __future__ import annotations

import os
import sys

import numpy as np

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__)))))
from logkv_b200.workload import MixtureKeys, apply_rope, boundary_pattern, rope_tables  # noqa: E402

BASE = dict(batch=2, groups=2, dim=16, clusters=4, slots=16, recent=32, granularity=32,
            exact=8, span_cap=4, beta=True, max_seq=512, chunk=32, steps=14, dtype="fp32",
            sigma=0.3, orphan_frac=0.08, boundaries="mixed", outliers=True, jumps=False, seed=0)

CONFIGS = [
    dict(BASE, name="fp32_beta"),
    dict(BASE, name="fp32_alpha", beta=False, seed=1),
    dict(BASE, name="bf16_beta", dtype="bf16", seed=2),
    dict(BASE, name="fp32_beta_sh", s_h=3.0, seed=3, jumps=True),
    dict(BASE, name="fp32_beta_g2k", granularity=16, recent=32, chunk=24, steps=18, seed=4),
    dict(BASE, name="bf16_beta_ropebf16", dtype="bf16", rope_dtype="bf16", seed=5, clusters=6, slots=12),
]


# Unified (Ward / radius) route variants: the same miniature streams with
# semantic_unified_route=True.  The default radius (s_h = 1) lets nearby tokens
# form candidates; s_h = 3 widens it; merge_passes = 2 adds frozen-centre sweeps
# to the global pass.
UNIFIED_CONFIGS = [
    dict(BASE, name="fp32_unified", unified=True, seed=6),
    dict(BASE, name="bf16_unified", dtype="bf16", unified=True, seed=7),
    dict(BASE, name="fp32_unified_sh", unified=True, s_h=3.0, seed=8, jumps=True),
    dict(BASE, name="fp32_unified_passes2", unified=True, merge_passes=2, seed=9),
    dict(BASE, name="bf16_unified_nobeta", dtype="bf16", unified=True, beta=False, merge_passes=3, seed=10,
         clusters=6, slots=12),
    # Wider flushes (96 tokens, head dim 32): the candidate and global passes take the Gram form.
    dict(BASE, name="fp32_unified_wide", unified=True, recent=96, granularity=96, chunk=96, steps=9,
         max_seq=1024, dim=32, clusters=6, exact=16, span_cap=8, seed=11),
    dict(BASE, name="bf16_unified_wide", dtype="bf16", unified=True, recent=96, granularity=96, chunk=96,
         steps=9, max_seq=1024, dim=32, clusters=6, exact=16, span_cap=8, s_h=2.0, merge_passes=2, seed=12),
]


def make_stream(cfg: dict) -> dict:
    rng = np.random.default_rng(cfg["seed"])
    Bt, G, D, T = cfg["batch"], cfg["groups"], cfg["dim"], cfg["chunk"]
    mix = MixtureKeys(rng, G, D, cfg["clusters"], sigma=cfg["sigma"], orphan_frac=cfg["orphan_frac"])
    cos, sin = rope_tables(cfg["max_seq"] + 64, D)
    chunks = []
    pos_next = np.zeros(Bt, dtype=np.int64)
    for step in range(cfg["steps"]):
        k_raw = mix.draw(Bt, T)
        if cfg["outliers"]:
            for b in range(Bt):
                if rng.random() < 0.7:
                    length = int(rng.integers(1, cfg["span_cap"] + 1))
                    start = int(rng.integers(0, T - length + 1))
                    mix.plant_outlier_span(k_raw, b, start, length, float(rng.uniform(3.0, 9.0)))
        v = rng.standard_normal((Bt, G, T, D)).astype(np.float32)
        q = rng.standard_normal((Bt, 2 * G, T, D)).astype(np.float32)
        if cfg["jumps"]:
            steps_ = 1 + (rng.random((Bt, T)) < 0.1) * rng.integers(1, 4, size=(Bt, T))
            pos = pos_next[:, None] + np.cumsum(steps_, axis=1) - steps_[:, :1]
            pos_next = pos[:, -1] + 1
        else:
            pos = pos_next[:, None] + np.arange(T)[None, :]
            pos_next = pos[:, -1] + 1
        if cfg["boundaries"] == "mixed":
            ends = np.stack([boundary_pattern(rng, 1, T, "mod3")[0] if b % 2 == 0
                             else boundary_pattern(rng, 1, T, "random")[0] for b in range(Bt)])
        else:
            ends = boundary_pattern(rng, Bt, T, cfg["boundaries"])
        k = apply_rope(k_raw, pos[:, None, :], cos, sin)
        chunks.append(dict(k=k, k_raw=k_raw, v=v, q=q, pos=pos if cfg["jumps"] else None,
                           positions=pos, span_ends=ends, attend=step % 3 == 2))
    return dict(cos=cos, sin=sin, chunks=chunks)
