"""Decode attention at the decode benchmark's cache shape against the float64 oracle.

The cache is the benchmark's (BASELINE configs[3] layer shape, batch 8): 8 KV groups x 128, 12
clusters x 4 full levels x B'=125 merged slots with Geometric(0.1) counts and mid anchors (6000
pooled slots per lane), 256 exact rows, a full 2048-token window.  A decode step's attention is
compared with the oracle's packer and float64 softmax, within the bf16 tolerance of the flush and
attention parity tests: a single new token (causal), and the reference's paired step, where the
one query of the current token also sees the pending token (two new keys, causal_tail=0,
litgpt/model.py:1219-1226).
"""
from __future__ import annotations

import os
import sys

import numpy as np
import pytest
import torch

from oracle import attention as A

pytestmark = pytest.mark.gpu
TOL = 2e-2
ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def oracle(cache, cos, sin, q, k, v, causal_tail):
    h = lambda t: t.detach().float().cpu().numpy() if t.dtype == torch.bfloat16 else t.detach().cpu().numpy()  # noqa
    plan = A.mid_plan(h(cache.level_count), h(cache.level_w), h(cache.level_sum_wp))
    D = cache.k_dim
    ka, va = A.pack_mid(h(cache.level_k), h(cache.level_v), h(cache.level_w), plan, h(cache.alpha_k_raw),
                        h(cache.alpha_v), h(cache.alpha_pos), h(cache.alpha_valid), cache.alpha_count,
                        h(cache.recent_k), h(cache.recent_v), cache.recent_count, h(k), h(v), cos, sin, D,
                        ((D + 8) // 8) * 8, "bf16", "fp32")
    return A.slot_attention(h(q), ka, va, D ** -0.5, causal_tail, D, "bf16")


@pytest.mark.parametrize("new_keys", [1, 2])
def test_decode_at_benchmark_shape_matches_oracle(new_keys):
    sys.path.insert(0, ROOT)
    from bench import DECODE, prefill_decode_cache
    from logkv_b200 import log_kv_chunk_attention
    from logkv_b200.workload import rope_tables
    cfg = dict(DECODE)
    batch, H, G, D = 8, cfg["heads"], cfg["groups"], cfg["head_dim"]
    cos_np, sin_np = rope_tables(cfg["max_seq"] + 1024, D, base=1e6)
    cos, sin = torch.from_numpy(cos_np).cuda(), torch.from_numpy(sin_np).cuda()
    cache = prefill_decode_cache(torch, cfg, batch, torch.device("cuda"), cos, sin, seed=11)
    assert int(cache.level_count.sum(-1).float().mean().item()) == 4 * cache.B_prime
    gen = torch.Generator(device="cuda").manual_seed(5 + new_keys)
    q = torch.randn(batch, H, 1, D, generator=gen, device="cuda").bfloat16()
    k = torch.randn(batch, G, new_keys, D, generator=gen, device="cuda").bfloat16()
    v = torch.randn(batch, G, new_keys, D, generator=gen, device="cuda").bfloat16()
    causal_tail = 1 if new_keys == 1 else 0
    with torch.no_grad():
        out = log_kv_chunk_attention(cache, q, k, v, D ** -0.5, 0.0, causal_tail=causal_tail, reuse_prefix=True)
    torch.cuda.synchronize()
    assert int(cache._read.status.item()) == 0
    assert out.shape == (batch, H, 1, D)
    if new_keys == 2:
        # The oracle's causal-tail form takes equal query and key counts: pad the query block with a
        # second (ignored) row; with causal_tail=0 every row sees both new keys.
        q2 = torch.cat([q, q], dim=2)
        want = oracle(cache, cos_np, sin_np, q2, k, v, 0)[:, :, :1]
    else:
        want = oracle(cache, cos_np, sin_np, q, k, v, 1)
    err = np.abs(out.float().cpu().numpy() - want).max()
    assert err <= TOL, err
