"""Operator-level plugin functions on the GPU against the oracle, on seeded inputs.

Each function of ``logkv_b200.plugin`` (the reference's fused-kernel module API,
log_kv_updates_triton.py / log_kv_route_triton.py / log_kv_pack_triton.py) must equal
the oracle's restatement of the reference's CPU arithmetic bit for bit.
"""
from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle.attach import attach_assign_kernel
from oracle.ladder import Rows, beta_layout, beta_merge, merge_pairs
from oracle.numerics import F32, seq_sum, to_storage

pytestmark = pytest.mark.gpu

DEV = "cuda"


def fields_of(n, dk, dv, dtype, gen, *, kv=True):
    """A reference 13-field tuple of n random rows on the GPU (None for the unused fields)."""
    f = [None] * 13
    f[0] = torch.randn(n, dk, generator=gen).to(DEV, dtype)
    f[1] = torch.randn(n, dv, generator=gen).to(DEV, dtype)
    f[2] = torch.randint(0, 5, (n,), generator=gen).float().to(DEV)
    pos = torch.randint(0, 1000, (n,), generator=gen)
    f[8] = pos.to(DEV)
    f[9] = (pos + torch.randint(0, 9, (n,), generator=gen)).to(DEV)
    f[10] = (pos * 3).to(DEV)
    f[11] = torch.randint(0, 50, (n,), generator=gen).to(DEV)
    f[12] = (torch.rand(n, generator=gen) < 0.2).to(DEV)
    return f


def host_rows(f, idx=None) -> Rows:
    t = lambda x: x.detach().cpu().float().numpy() if x.dtype == torch.bfloat16 else x.detach().cpu().numpy()  # noqa
    r = Rows(t(f[0]).astype(F32), t(f[1]).astype(F32), t(f[2]).astype(F32), t(f[8]), t(f[9]), t(f[10]), t(f[11]),
             t(f[12]).astype(bool))
    return r if idx is None else r.take(idx)


def assert_rows_equal(got: Rows, want: Rows, msg=""):
    for a, b, name in zip(got.fields(), want.fields(), ("k", "v", "w", "lo", "hi", "swp", "order", "pad")):
        np.testing.assert_array_equal(np.asarray(a), np.asarray(b), err_msg=f"{msg} {name}")


def test_fill_casts_staged_rows():
    from logkv_b200 import plugin
    gen = torch.Generator().manual_seed(1)
    fields = fields_of(40, 16, 16, torch.bfloat16, gen)
    stage = fields_of(12, 16, 16, torch.float32, gen)
    src = torch.tensor([3, 0, 11, 7], device=DEV)
    dst = torch.tensor([39, 2, 5, 20], device=DEV)
    before = host_rows(fields)
    plugin.fill(fields, stage, src, dst)
    torch.cuda.synchronize()
    got = host_rows(fields)
    want = before
    s = host_rows(stage).take(src.cpu().numpy()).cast("bf16")
    for name_i, arr in enumerate(want.fields()):
        arr[dst.cpu().numpy()] = s.fields()[name_i]
    assert_rows_equal(got, want, "fill")


@pytest.mark.parametrize("beta", [False, True])
def test_merge_scatter_matches_oracle(beta):
    from logkv_b200 import plugin
    gen = torch.Generator().manual_seed(2 + beta)
    dk = dv = 32
    fields = fields_of(60, dk, dv, torch.bfloat16, gen)
    stage = fields_of(20, dk, dv, torch.float32, gen)
    si = torch.randperm(60, generator=gen)[:30].to(DEV)
    gi = torch.randperm(20, generator=gen)[:14].to(DEV)
    pool_host = Rows.cat(host_rows(fields, si.cpu().numpy()), host_rows(stage, gi.cpu().numpy()).cast("bf16"))
    lengths = [8, 6, 2, 12] if beta else None
    npi = sum(lengths) if beta else 20
    perm = torch.randperm(44, generator=gen)
    pi = perm[:npi].to(DEV)
    vi = perm[npi:npi + 6].to(DEV)
    dst = torch.tensor([50, 51, 52, 53, 54, 55], device=DEV)
    clear = torch.tensor([56, 57], device=DEV)
    before = host_rows(fields)
    pristine = [None if t is None else t.clone() for t in fields]
    if beta:
        carry, cuts = plugin.merge_scatter(fields, stage, si, gi, pi, vi, dst, clear, beta_lengths=lengths)
    else:
        carry = plugin.merge_scatter(fields, stage, si, gi, pi, vi, dst, clear)
    torch.cuda.synchronize()
    pool_pi = pool_host.take(pi.cpu().numpy())
    if beta:
        parts, all_cuts, base = [], [], 0
        for n in lengths:
            merged, c = beta_merge(pool_pi.take(slice(base, base + n)))
            parts.append(merged)
            all_cuts.extend(np.asarray(c).tolist())
            base += n
        want = parts[0]
        for p in parts[1:]:
            want = Rows.cat(want, p)
        assert cuts.cpu().tolist() == all_cuts
        assert beta_layout(lengths).shape[0] == len(all_cuts)
    else:
        want = merge_pairs(pool_pi)
    assert_rows_equal(host_rows(carry), want, "carry")
    if beta:   # replaying the recorded cuts gives the same carry
        carry2, _ = plugin.merge_scatter(pristine, stage, si, gi, pi, vi, dst, clear[:0], beta_lengths=lengths,
                                         beta_cuts=cuts.clone())
        assert_rows_equal(host_rows(carry2), want, "replay")
    got = host_rows(fields)
    surv = pool_host.take(vi.cpu().numpy())
    for i, arr in enumerate(before.fields()):
        arr[dst.cpu().numpy()] = surv.fields()[i]
        arr[clear.cpu().numpy()] = 0
    assert_rows_equal(got, before, "scatter")


def test_centroid_ordered_runs():
    from logkv_b200 import plugin
    gen = torch.Generator().manual_seed(4)
    D, C = 24, 6
    k = torch.randn(50, D, generator=gen).to(DEV, torch.bfloat16)
    mu = torch.randn(C, D, generator=gen).to(DEV)
    ne = torch.tensor([0., 3., 1.5, 0., 7., 2.], device=DEV)
    forget = np.asarray([1.0, 0.5, 1.0, 1.0], F32).view(np.int32).astype(np.int64)
    meta = torch.tensor([[1, 4, 0, 5], [0, 0, 0, 0], [0, 10, 22, 40], [10, 12, 18, 10], forget.tolist()],
                        dtype=torch.int64, device=DEV)
    mu0, ne0, kh = mu.cpu().numpy().copy(), ne.cpu().numpy().copy(), k.float().cpu().numpy()
    plugin.centroid(k, mu, ne, meta, 0, 4)
    torch.cuda.synchronize()
    want_mu, want_ne = mu0.copy(), ne0.copy()
    m = meta.cpu().numpy()
    for r in range(4):
        c, begin, n = m[0, r], m[2, r], m[3, r]
        f = np.asarray([m[4, r]], np.int64).astype(np.int32).view(F32)[0]
        acc = seq_sum(kh[begin:begin + n])
        pre = F32(ne0[c] * f)
        denom = F32(pre + F32(n))
        want_mu[c] = ((pre * mu0[c]).astype(F32) + acc).astype(F32) / denom if pre > 0 else acc / F32(n)
        want_ne[c] = denom
    np.testing.assert_array_equal(mu.cpu().numpy(), want_mu.astype(F32))
    np.testing.assert_array_equal(ne.cpu().numpy(), want_ne)


def test_alpha_partition_gathers():
    from logkv_b200 import plugin
    gen = torch.Generator().manual_seed(5)
    B, G, N, D, P, A = 2, 3, 20, 16, 6, 9
    k = torch.randn(B, G, N, D, generator=gen).to(DEV, torch.bfloat16)
    v = torch.randn(B, G, N, D, generator=gen).to(DEV, torch.bfloat16)
    pos = torch.randint(0, 999, (B, N), generator=gen).to(DEV)
    idx = torch.full((B, P + A), -1, dtype=torch.int64)
    for b in range(B):
        perm = torch.randperm(N, generator=gen)
        idx[b, :P - 1] = perm[:P - 1]
        idx[b, P:P + A - 2] = perm[P:P + A - 2]
    idx = idx.to(DEV)
    ek, ev = torch.zeros(B, G, P, D, dtype=torch.bfloat16, device=DEV), torch.zeros(B, G, P, D, dtype=torch.bfloat16, device=DEV)
    ep, valid = torch.zeros(B, P, dtype=torch.int64, device=DEV), torch.zeros(B, P, dtype=torch.bool, device=DEV)
    ak, av, ap = plugin.alpha_partition(k, v, pos, idx, (ek, ev, ep, valid))
    torch.cuda.synchronize()
    ih = idx.cpu().numpy()
    kh, vh, ph = k.float().cpu().numpy(), v.float().cpu().numpy(), pos.cpu().numpy()
    for b in range(B):
        for row in range(P + A):
            s = ih[b, row]
            want_k = kh[b, :, s] if s >= 0 else np.zeros((G, D), F32)
            want_v = vh[b, :, s] if s >= 0 else np.zeros((G, D), F32)
            if row < P:
                np.testing.assert_array_equal(ek[b, :, row].float().cpu().numpy(), want_k)
                np.testing.assert_array_equal(ev[b, :, row].float().cpu().numpy(), want_v)
                assert ep[b, row].item() == (ph[b, s] if s >= 0 else 0)
                assert valid[b, row].item() == (s >= 0)
            else:
                np.testing.assert_array_equal(ak[b, :, row - P].float().cpu().numpy(), want_k)
                np.testing.assert_array_equal(av[b, :, row - P].float().cpu().numpy(), want_v)
                assert ap[b, row - P].item() == (ph[b, s] if s >= 0 else 0)


def test_attach_assign_matches_oracle():
    from logkv_b200 import plugin
    rng = np.random.default_rng(6)
    B, G, T, D, K = 2, 3, 40, 32, 6
    centres = rng.standard_normal((B, G, K, D)).astype(F32)
    x = (centres[:, :, rng.integers(0, K, T)].transpose(0, 1, 2, 3) +
         0.4 * rng.standard_normal((B, G, T, D))).astype(F32)
    x = to_storage(x, "bf16")
    pos = np.stack([rng.permutation(1000)[:T] for _ in range(B)]).astype(np.int64)
    order = np.argsort(pos, axis=1, kind="stable").astype(np.int64)
    counts = np.asarray([T, T - 7], np.int64)
    alive = rng.random((B, G, K)) < 0.8
    p_hi = rng.integers(0, 800, (B, G, K)).astype(np.int64)
    s_h = rng.uniform(5, 60, (B, G)).astype(F32)
    want = attach_assign_kernel(x, pos, order, counts, centres, alive, p_hi, s_h, 1.0, 2048.0, 1.0)
    t = lambda a, dt=None: torch.from_numpy(np.ascontiguousarray(a)).to(DEV) if dt is None else torch.from_numpy(a).to(DEV, dt)  # noqa
    got = plugin.attach_assign(t(x, torch.bfloat16), t(pos), t(order), t(counts), t(centres), t(alive), t(p_hi), t(s_h),
                               1.0, 2048.0, 1.0)
    np.testing.assert_array_equal(got.cpu().numpy(), want)


def test_pack_on_a_cache_with_only_the_reference_buffers():
    """plugin.pack through the adapter (only the reference's buffer names) equals pack_mid_kv."""
    import types
    from fixtures import config, make_stream
    from test_flush_gpu import make_cache, push_chunk
    from logkv_b200 import plugin
    from logkv_b200.attention import pack_mid_kv
    cfg = config("bf16_beta")
    stream = make_stream(cfg)
    cache = make_cache(cfg, stream)
    for chunk in stream["chunks"][:5]:
        push_chunk(cache, cfg, chunk)
    names = ["level_k", "level_v", "level_w", "level_sum_wp", "level_count", "recent_k", "recent_v", "alpha_k_raw",
             "alpha_v", "alpha_pos", "alpha_valid", "cos_cache", "sin_cache", "batch_size", "n_groups", "k_dim",
             "v_dim", "K_max", "L_alloc", "B_prime", "alpha_exact_tokens", "alpha_count", "recent_count",
             "rope_n_elem", "semantic_pack_backend", "semantic_anchor_mode"]
    foreign = types.SimpleNamespace(**{n: getattr(cache, n) for n in names})
    chunk = stream["chunks"][5]
    k = torch.from_numpy(chunk["k"]).to(DEV, torch.bfloat16)
    v = torch.from_numpy(chunk["v"]).to(DEV, torch.bfloat16)
    plan = cache._semantic_attention_plan()
    a_k, a_v = plugin.pack(foreign, plan, k, v, 24)
    b_k, b_v = pack_mid_kv(cache, plan, k, v, 24)
    torch.testing.assert_close(a_k, b_k, atol=0, rtol=0)
    torch.testing.assert_close(a_v, b_v, atol=0, rtol=0)
