"""Full-size device flush against the oracle: the benchmark's layer shape, bit for bit.

8 KV groups x 128, K=12, B=128 (B'=125), window 2048, 2048-token flushes,
exact pool 256 with 64-token spans, Beta on, bf16.  Planted outlier spans make
Alpha evict older exact spans, so delayed re-inserts run at full size too.
Also checks the size-independent invariants of the reference's tests: token
mass and weighted K/V payload are conserved across ladder, exact pool and window.
"""
from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle.cache import OracleCache

pytestmark = pytest.mark.gpu

G, D, K, T = 8, 128, 12, 2048


def stream(n_chunks, seed=3):
    from logkv_b200.workload import MixtureKeys, boundary_pattern
    rng = np.random.default_rng(seed)
    mix = MixtureKeys(rng, G, D, K)
    out = []
    for c in range(n_chunks):
        kr = mix.draw(1, T)
        for _ in range(3):
            length = int(rng.integers(8, 65))
            start = int(rng.integers(0, T - length))
            mix.plant_outlier_span(kr, 0, start, length, float(rng.uniform(4.0, 12.0)))
        v = rng.standard_normal((1, G, T, D)).astype(np.float32)
        pos = np.arange(c * T, (c + 1) * T)[None]
        ends = boundary_pattern(rng, 1, T, "mod23")
        out.append((kr, v, pos, ends))
    return out


def test_fullsize_flush_matches_oracle(cascade_path):
    from logkv_b200.cache import LogStructuredKVCache
    from logkv_b200.workload import rope_tables
    cos, sin = rope_tables(32768, D, base=1e6)
    cache = LogStructuredKVCache((1, G, 32768, D), (1, G, 32768, D), B=128, recent_size=2048, device="cuda",
                                 dtype=torch.bfloat16, semantic_clusters=True, semantic_anchor_mode="mid",
                                 allocate_second_order=False, cluster_k_max=K, semantic_flush_granularity=2048,
                                 alpha_exact_tokens=256, alpha_span_max_tokens=64, beta_novelty=True,
                                 beta_adaptive_merge=True, cos_cache=torch.from_numpy(cos),
                                 sin_cache=torch.from_numpy(sin), rope_n_elem=D)
    oc = OracleCache(batch=1, groups=G, max_seq=32768, dim=D, B=128, recent=2048, clusters=K, granularity=2048,
                     exact=256, span_cap=64, beta=True, dtype="bf16")
    source_sum = np.zeros((G, D), np.float64)
    for step, (kr, v, pos, ends) in enumerate(stream(4)):
        k_t = torch.from_numpy(kr).to("cuda", torch.bfloat16)
        v_t = torch.from_numpy(v).to("cuda", torch.bfloat16)
        cache.add_recent(k_t, v_t, k_raw=k_t, span_ends=ends.tolist())
        oc.add_recent(kr, v, kr, pos, ends)
        source_sum += k_t.float().cpu().numpy()[0].sum(1)
        assert cache.read_status() == 0
        st = oc.state()
        for name, want in st.items():
            got = getattr(cache, name).detach().cpu()
            got = got.float().numpy() if got.dtype == torch.bfloat16 else got.numpy()
            np.testing.assert_array_equal(got.astype(want.dtype), want, err_msg=f"step {step} {name}")
        assert cache._alpha_spans == [[(int(a), bool(c)) for a, c in row] for row in oc.alpha_spans]
        # Mass and payload conservation (reference tests/test_alpha_log_kv.py:119-160).
        mass = cache.level_w.sum((2, 3, 4)) + cache.alpha_valid.sum(-1)[:, None] + cache.recent_count
        assert torch.equal(mass.cpu(), torch.full_like(mass.cpu(), (step + 1) * T))
        total = (cache.level_k.float() * cache.level_w[..., None]).sum((2, 3, 4))
        total += (cache.alpha_k_raw.float() * cache.alpha_valid[:, None, :, None]).sum(2)
        total += cache.recent_k_raw[:, :, :cache.recent_count].float().sum(2)
        np.testing.assert_allclose(total[0].cpu().numpy(), source_sum, atol=0.5, rtol=0.02)
    counters = cache.read_counters()
    assert counters["flushes"] == 3 and counters["survivor"] > 0
