"""Seeded full-shape flush cases (the single-layer CPU configuration of the flush benchmark).

One layer's cache at the production geometry: batch 1, 8 KV groups, head dim 128,
K = 12 clusters, B = 128 slots (B' = 125 after the 256-token exact pool), a
2048-token recent window flushed 2048 tokens at a time, 64-token span cap, Beta
on, mid anchors.  Keys come from a 12-component isotropic Gaussian mixture per
group (centres ~ N(0, 1), within-cluster sigma 0.3) with 5% orphans far from
every centre and two planted 32-token outlier spans per flushed chunk; span
boundaries every 16th token and at every planted span's end; V ~ N(0, 1).

Chunk 0 fills the window without flushing.  Then a pre-state is planted in
the cluster table (``plant``): the first ``alive`` clusters of every lane are
alive with their centroid at the mixture centre, n_eff = n_total = 128 and
p_hi_c just before the window; the ladder stays empty.  Chunks 1..3 each
trigger one 2048-token flush.  The cases vary the storage dtype, the direct
join threshold s_h (1: every token takes the nearest-exact branch; 12: the
threshold falls inside the within-cluster distance distribution; 32: nearly
every token joins directly) and the number of alive clusters (8 of 12: the
remaining 4 are opened by farthest-point seeding on the first flush).

Shared by ``make_fullshape.py`` (runs the reference) and the tests.
"""
from __future__ import annotations

import os
import sys

import numpy as np

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__)))))
from logkv_b200.workload import MixtureKeys, apply_rope, rope_tables  # noqa: E402

GEOM = dict(batch=1, groups=8, dim=128, clusters=12, slots=128, recent=2048, granularity=2048, exact=256,
            span_cap=64, beta=True, max_seq=32768, chunk=2048, chunks=4, sigma=0.3, orphan_frac=0.05,
            start=4096, rope_base=1e6, prestate_count=128)

CASES = [
    dict(GEOM, name="f32_sh1", dtype="fp32", s_h=1.0, alive=12, seed=10),
    dict(GEOM, name="f32_sh12", dtype="fp32", s_h=12.0, alive=12, seed=11),
    dict(GEOM, name="f32_sh32", dtype="fp32", s_h=32.0, alive=12, seed=12),
    dict(GEOM, name="f32_seed", dtype="fp32", s_h=1.0, alive=8, seed=13),
    dict(GEOM, name="bf16_sh1", dtype="bf16", s_h=1.0, alive=12, seed=14),
    dict(GEOM, name="bf16_seed", dtype="bf16", s_h=12.0, alive=8, seed=15),
]


# The unified (Ward / radius) route at the same shape: radius sqrt(s_h) = 1 (few candidates
# merge: the global pass reduces ~2300 rows), sqrt(32) (candidates absorb most tokens), and
# frozen-centre sweeps in the global pass.
UNIFIED_CASES = [
    dict(GEOM, name="f32_unified", dtype="fp32", s_h=1.0, alive=12, seed=20, unified=True),
    dict(GEOM, name="bf16_unified_sh32", dtype="bf16", s_h=32.0, alive=8, seed=21, unified=True),
    dict(GEOM, name="f32_unified_passes2", dtype="fp32", s_h=4.0, alive=12, seed=22, unified=True, merge_passes=2),
]


def case(name: str) -> dict:
    return next(c for c in CASES + UNIFIED_CASES if c["name"] == name)


def make_case(cfg: dict) -> dict:
    """Inputs of one case: RoPE tables, the mixture centres and the chunks (float32 numpy)."""
    rng = np.random.default_rng(cfg["seed"])
    B, G, D, T = cfg["batch"], cfg["groups"], cfg["dim"], cfg["chunk"]
    mix = MixtureKeys(rng, G, D, cfg["clusters"], sigma=cfg["sigma"], orphan_frac=cfg["orphan_frac"])
    cos, sin = rope_tables(cfg["max_seq"], D, base=cfg["rope_base"])
    chunks = []
    for c in range(cfg["chunks"]):
        k_raw = mix.draw(B, T)
        ends = (np.arange(T) % 16) == 15
        ends = np.broadcast_to(ends, (B, T)).copy()
        if c > 0:
            for start in rng.choice(np.arange(1, T // 32 - 1), size=2, replace=False) * 32:
                mix.plant_outlier_span(k_raw, 0, int(start), 32, 6.0)
                ends[:, int(start) + 31] = True
        v = rng.standard_normal((B, G, T, D)).astype(np.float32)
        pos = cfg["start"] + c * T + np.arange(T, dtype=np.int64)
        k = apply_rope(k_raw, np.broadcast_to(pos, (B, G, T)), cos, sin)
        chunks.append(dict(k=k, k_raw=k_raw, v=v, pos=pos, span_ends=ends))
    return dict(cos=cos, sin=sin, centres=mix.centres, chunks=chunks)


def prestate(cfg: dict, inputs: dict) -> dict:
    """Cluster-table values planted after chunk 0 (numpy, the buffers' dtypes)."""
    B, G, K, D = cfg["batch"], cfg["groups"], cfg["clusters"], cfg["dim"]
    alive = np.zeros((B, G, K), dtype=bool)
    alive[:, :, :cfg["alive"]] = True
    centroid = np.zeros((B, G, K, D), dtype=np.float32)
    centroid[:, :, :cfg["alive"]] = inputs["centres"][None, :, :cfg["alive"]]
    n = cfg["prestate_count"]
    return dict(alive=alive, centroid=centroid,
                n_eff=np.where(alive, np.float32(n), np.float32(0)).astype(np.float32),
                n_total=np.where(alive, n, 0).astype(np.int32),
                p_hi_c=np.where(alive, cfg["start"] - 1, -1).astype(np.int64),
                level0_phase=np.where(alive, n, 0).astype(np.int32))


# Per-(b, g, k, l) digests of the level K/V rows: an exact bit hash (equal iff every stored bit
# is equal) and float64 projections on fixed +-1 vectors (for tolerance checks).
def bit_hash(bits: np.ndarray) -> np.ndarray:
    """bits [..., rows, D] (uint16 or uint32 patterns) -> uint64 [...] position-weighted hash."""
    lead = bits.shape[:-2]
    flat = bits.reshape(*lead, -1).astype(np.uint64)
    weights = (np.arange(flat.shape[-1], dtype=np.uint64) * np.uint64(2654435761) + np.uint64(1)) | np.uint64(1)
    with np.errstate(over="ignore"):
        mixed = (flat + np.uint64(0x9E3779B97F4A7C15)) * weights
        mixed ^= mixed >> np.uint64(29)
        return mixed.sum(axis=-1, dtype=np.uint64)


def projections(values: np.ndarray, seed: int = 1234) -> np.ndarray:
    """values [..., rows, D] float -> float64 [..., 3]: sum, and two fixed +-1 projections."""
    D = values.shape[-1]
    rng = np.random.default_rng(seed)
    r = np.stack([np.ones(D), rng.choice([-1.0, 1.0], D), rng.choice([-1.0, 1.0], D)], axis=1)
    v = values.astype(np.float64)
    return np.einsum("...rd,dp->...p", v, r)
