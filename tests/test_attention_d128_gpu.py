"""Head-dim-128 attention kernels (decode split-K on mma.sync, chunk on tcgen05/TMEM) vs the oracle.

The golden streams use head dim 16; these cases write a D=128 bf16 cache directly
(full merged levels with Geometric(0.1) counts and mid anchors, an exact pool, a
window) and compare decode (1 and 2 tokens) and chunk attention (300 tokens, so the
last 128-row query tile is partial) with the float64 oracle over the same state.
"""
from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import attention as A
from oracle.numerics import to_storage

pytestmark = pytest.mark.gpu

TOL = 2e-2


def make_state(seed=0, B=1, G=2, D=128, K=4, levels=3, recent=512, R=300, P=64, max_seq=8192):
    from logkv_b200.cache import LogStructuredKVCache
    from logkv_b200.workload import rope_tables
    cos, sin = rope_tables(max_seq + 64, D, base=1e6)
    cache = LogStructuredKVCache(
        (B, G, max_seq, D), (B, G, max_seq, D), B=32, recent_size=recent, device="cuda", dtype=torch.bfloat16,
        semantic_clusters=True, semantic_anchor_mode="mid", allocate_second_order=False,
        cluster_k_max=K, semantic_flush_granularity=recent, alpha_exact_tokens=P, alpha_span_max_tokens=16,
        beta_novelty=True, beta_adaptive_merge=True, cos_cache=torch.from_numpy(cos), sin_cache=torch.from_numpy(sin),
        rope_n_elem=D)
    gen = torch.Generator(device="cuda").manual_seed(seed)
    lv = (slice(None), slice(None), slice(None), slice(0, levels))
    Bs = cache.B_prime
    cache.level_k[lv].normal_(generator=gen)
    cache.level_v[lv].normal_(generator=gen)
    u = torch.rand(cache.level_w[lv].shape, generator=gen, device="cuda").clamp_min(1e-7)
    w = torch.floor(torch.log(u) / np.log(0.9)) + 1.0
    m = torch.randint(0, max_seq, w.shape, generator=gen, device="cuda")
    cache.level_w[lv] = w
    cache.level_sum_wp[lv] = w.long() * m
    cache.level_count[:, :, :, :levels] = Bs
    cache.level_count[0, 0, 1, 2] = Bs // 3          # ragged lanes
    cache.level_w[0, min(1, G - 1), 0, 0, 5] = 0.0   # an occupied slot with zero weight (invalid)
    cache.alpha_k_raw.normal_(generator=gen)
    cache.alpha_v.normal_(generator=gen)
    cache.alpha_pos.copy_(torch.randint(0, max_seq, cache.alpha_pos.shape, generator=gen, device="cuda"))
    cache.alpha_valid.fill_(True)
    cache.alpha_valid[0, 3] = False
    cache._row_count.fill_(P)
    cache._alpha_count_dev.fill_(P)
    cache.recent_k[:, :, :R].normal_(generator=gen)
    cache.recent_v[:, :, :R].normal_(generator=gen)
    cache.recent_count = R
    cache._ladder_epoch += 1
    return cache, cos, sin


def oracle(cache, cos, sin, q, k, v):
    h = lambda t: t.detach().float().cpu().numpy() if t.dtype == torch.bfloat16 else t.detach().cpu().numpy()  # noqa
    plan = A.mid_plan(h(cache.level_count), h(cache.level_w), h(cache.level_sum_wp))
    D = cache.k_dim
    ka, va = A.pack_mid(h(cache.level_k), h(cache.level_v), h(cache.level_w), plan, h(cache.alpha_k_raw),
                        h(cache.alpha_v), h(cache.alpha_pos), h(cache.alpha_valid), cache.alpha_count,
                        h(cache.recent_k), h(cache.recent_v), cache.recent_count, h(k), h(v), cos, sin, D,
                        ((D + 8) // 8) * 8, "bf16", "fp32")
    return A.slot_attention(h(q), ka, va, D ** -0.5, q.size(2), D, "bf16")


@pytest.mark.parametrize("T", [1, 2, 300])
def test_d128_attention_matches_oracle(T):
    from logkv_b200 import log_kv_chunk_attention
    cache, cos, sin = make_state(seed=T)
    gen = torch.Generator(device="cuda").manual_seed(100 + T)
    q = torch.randn(1, 4, T, 128, generator=gen, device="cuda").bfloat16()
    k = torch.randn(1, 2, T, 128, generator=gen, device="cuda").bfloat16()
    v = torch.randn(1, 2, T, 128, generator=gen, device="cuda").bfloat16()
    with torch.no_grad():
        out = log_kv_chunk_attention(cache, q, k, v, 128 ** -0.5, 0.0)
    torch.cuda.synchronize()
    assert int(cache._read.status.item()) == 0
    want = oracle(cache, cos, sin, q, k, v)
    err = np.abs(out.float().cpu().numpy() - want).max()
    assert err <= TOL, err
    if T > 2:   # the chunk kernel reports timeouts in the workspace status word
        ws = cache._read.workspaces[(4, T)]
        assert int(ws[:4].view(torch.int32).item()) == 0


@pytest.mark.parametrize("G", [8, 4, 2, 1])
def test_two_tile_chunk_kernel_matches_fp32_reference(G):
    """A 2048-token chunk (the two-tile tcgen05 kernel) against a PyTorch float32 softmax over
    the same packed K/V (the oracle's packer): 8 groups (128 query-tile pairs, one CTA each), and
    4, 2 or 1 groups (a KV-head-sharded rank's share at 2, 4 or 8 ranks: the key range is split
    over several CTAs per pair and the splits combined)."""
    from logkv_b200 import log_kv_chunk_attention
    H, T, D = 2 * G, 2048, 128
    cache, cos, sin = make_state(seed=7, G=G, recent=512, R=300, max_seq=8192)
    gen = torch.Generator(device="cuda").manual_seed(77)
    q = torch.randn(1, H, T, D, generator=gen, device="cuda").bfloat16()
    k = torch.randn(1, G, T, D, generator=gen, device="cuda").bfloat16()
    v = torch.randn(1, G, T, D, generator=gen, device="cuda").bfloat16()
    scale = D ** -0.5
    with torch.no_grad():
        out = log_kv_chunk_attention(cache, q, k, v, scale, 0.0)
    torch.cuda.synchronize()
    assert int(cache._read.status.item()) == 0
    ws = cache._read.workspaces[(H, T)]
    assert int(ws[:4].view(torch.int32).item()) == 0
    h = lambda t: t.detach().float().cpu().numpy() if t.dtype == torch.bfloat16 else t.detach().cpu().numpy()  # noqa
    plan = A.mid_plan(h(cache.level_count), h(cache.level_w), h(cache.level_sum_wp))
    ka, va = A.pack_mid(h(cache.level_k), h(cache.level_v), h(cache.level_w), plan, h(cache.alpha_k_raw),
                        h(cache.alpha_v), h(cache.alpha_pos), h(cache.alpha_valid), cache.alpha_count,
                        h(cache.recent_k), h(cache.recent_v), cache.recent_count, h(k), h(v), cos, sin, D,
                        ((D + 8) // 8) * 8, "bf16", "fp32")
    kt = torch.from_numpy(np.asarray(ka, np.float32)).cuda()          # [1, G, S, 136]
    vt = torch.from_numpy(np.asarray(va, np.float32))[..., :D].cuda()  # [1, G, S, D]
    qa = torch.zeros(1, H, T, kt.shape[-1], device="cuda")
    qa[..., :D] = q.float()
    qa[..., D] = float(A.query_extra(scale, "bf16"))
    rf = H // G
    S = kt.shape[2]
    blocked = torch.arange(S, device="cuda")[None, :] > (S - T) + torch.arange(T, device="cuda")[:, None]
    worst = 0.0
    for hh in range(H):
        sc = scale * (qa[0, hh] @ kt[0, hh // rf].T)
        sc = sc.masked_fill(blocked, float("-inf"))
        ref = torch.softmax(sc, dim=-1) @ vt[0, hh // rf]
        worst = max(worst, (out[0, hh].float() - ref).abs().max().item())
    assert worst <= TOL, worst


@pytest.mark.parametrize("G", [8, 2])
def test_chunk_kernel_running_max_rescales(G):
    """Keys of the new chunk grow with their position (x (1 + t / 256)), so the running maximum of
    every query row rises unit after unit and the softmax rescales O many times while the next
    units' scores are already in flight; 8 groups (one CTA per query-tile pair) and 2 (the key
    range split over CTAs), against a PyTorch float32 softmax over the same packed K/V."""
    from logkv_b200 import log_kv_chunk_attention
    H, T, D = 2 * G, 2048, 128
    cache, cos, sin = make_state(seed=11, G=G, recent=512, R=300, max_seq=8192)
    gen = torch.Generator(device="cuda").manual_seed(78)
    q = torch.randn(1, H, T, D, generator=gen, device="cuda").bfloat16()
    grow = (1.0 + torch.arange(T, device="cuda", dtype=torch.float32) / 256.0)[None, None, :, None]
    k = (torch.randn(1, G, T, D, generator=gen, device="cuda") * grow).bfloat16()
    v = torch.randn(1, G, T, D, generator=gen, device="cuda").bfloat16()
    scale = D ** -0.5
    with torch.no_grad():
        out = log_kv_chunk_attention(cache, q, k, v, scale, 0.0)
    torch.cuda.synchronize()
    assert int(cache._read.status.item()) == 0
    assert int(cache._read.workspaces[(H, T)][:4].view(torch.int32).item()) == 0
    h = lambda t: t.detach().float().cpu().numpy() if t.dtype == torch.bfloat16 else t.detach().cpu().numpy()  # noqa
    plan = A.mid_plan(h(cache.level_count), h(cache.level_w), h(cache.level_sum_wp))
    ka, va = A.pack_mid(h(cache.level_k), h(cache.level_v), h(cache.level_w), plan, h(cache.alpha_k_raw),
                        h(cache.alpha_v), h(cache.alpha_pos), h(cache.alpha_valid), cache.alpha_count,
                        h(cache.recent_k), h(cache.recent_v), cache.recent_count, h(k), h(v), cos, sin, D,
                        ((D + 8) // 8) * 8, "bf16", "fp32")
    kt = torch.from_numpy(np.asarray(ka, np.float32)).cuda()
    vt = torch.from_numpy(np.asarray(va, np.float32))[..., :D].cuda()
    qa = torch.zeros(1, H, T, kt.shape[-1], device="cuda")
    qa[..., :D] = q.float()
    qa[..., D] = float(A.query_extra(scale, "bf16"))
    S = kt.shape[2]
    blocked = torch.arange(S, device="cuda")[None, :] > (S - T) + torch.arange(T, device="cuda")[:, None]
    worst = 0.0
    for hh in range(H):
        sc = scale * (qa[0, hh] @ kt[0, hh // 2].T)
        ref = torch.softmax(sc.masked_fill(blocked, float("-inf")), dim=-1) @ vt[0, hh // 2]
        worst = max(worst, (out[0, hh].float() - ref).abs().max().item())
    assert worst <= TOL, worst
