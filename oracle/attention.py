"""Mid-anchor attention plan, packing and slot attention (TEST INFRASTRUCTURE ONLY).

Restates, in numpy, the reference's read side of the compressed cache for the
in-scope configuration (mid anchors, first order, no segments):

  mid_plan        LogStructuredKVCache._semantic_mid_attention_plan  log_kv_cache.py:5979-6007
  rope_rows       _rotate_at_anchors                                  log_kv_position.py:74-101
  pack_mid        _pack_torch                                         log_kv_pack.py:27-72
  slot_attention  _slot_sdpa_inputs + SDPA with a lower-right causal
                  tail (_packed_flash_attention / log_kv_slot_attention)
                                                                      log_kv_cache.py:6439-6464, :6751-6758,
                                                                      :6802-6864

Integer outputs (plan indices, anchors, validity) and the packed K/V rows are
exact restatements; ``slot_attention`` evaluates the softmax in float64 from the
packed (storage-dtype) operands, so it is the high-precision value that both the
reference's CPU math path and the CUDA kernel approximate.
"""
from __future__ import annotations

import numpy as np

from .numerics import F32, round_bf16, to_storage


def mid_plan(count, w, sum_wp):
    """Occupied slots per lane, cluster-major with the top level first (log_kv_cache.py:5979-6007).

    count [B,G,K,L] (level_count), w [B,G,K,L,B'] float32 (level_w), sum_wp
    [B,G,K,L,B'] int64.  Returns (idx, anchors, valid) of shape [B,G,width]
    with width = the largest lane's occupied count; lanes shorter than width are
    padded with idx 0, anchor 0 and valid False, as the reference's
    ``clamp_min(0)`` / ``masked_fill`` leave them.
    """
    count = np.asarray(count, np.int64)
    B, G, K, L = count.shape
    Bs = w.shape[-1]
    lanes = []
    for b in range(B):
        for g in range(G):
            lane = []
            for c in range(K):
                for lv in range(L - 1, -1, -1):
                    start = (c * L + lv) * Bs
                    lane.extend(range(start, start + int(count[b, g, c, lv])))
            lanes.append(lane)
    width = max((len(x) for x in lanes), default=0)
    idx = np.zeros((B, G, width), np.int64)
    occupied = np.zeros((B, G, width), bool)
    for n, lane in enumerate(lanes):
        b, g = divmod(n, G)
        idx[b, g, :len(lane)] = lane
        occupied[b, g, :len(lane)] = True
    wf = np.asarray(w, F32).reshape(B, G, -1)
    sf = np.asarray(sum_wp, np.int64).reshape(B, G, -1)
    weights = np.take_along_axis(wf, idx, axis=2)
    sums = np.take_along_axis(sf, idx, axis=2)
    valid = occupied & (weights > 0)
    ww = np.maximum(np.trunc(weights).astype(np.int64), 1)          # weights.long().clamp_min(1)
    anchors = np.floor_divide(2 * sums + ww, 2 * ww)
    anchors = np.where(valid, anchors, 0)
    return idx, anchors, valid


def rope_rows(x, pos, cos, sin, rope_n: int, dtype: str, cos_dtype: str):
    """LitGPT RoPE of rows ``x[..., D]`` at integer positions ``pos[...]`` (log_kv_position.py:74-101).

    ``x`` holds storage-dtype values (float32 arrays, bf16-exact for 'bf16').
    Torch's type promotion decides the arithmetic: with a float32 operand on
    either side the products and the sum are float32 and the result is rounded
    once to the storage dtype; with bfloat16 content and bfloat16 tables every
    operation rounds to bfloat16.
    """
    x = np.asarray(x, F32)
    if rope_n == 0:
        return x.copy()
    half = rope_n // 2
    c = np.asarray(cos, F32)[pos][..., :rope_n]
    s = np.asarray(sin, F32)[pos][..., :rope_n]
    xr = x[..., :rope_n]
    rot = np.concatenate([-xr[..., half:], xr[..., :half]], axis=-1)
    if dtype == "bf16" and cos_dtype == "bf16":
        roped = round_bf16(round_bf16(xr * c) + round_bf16(rot * s))
    else:
        roped = to_storage((xr * c).astype(F32) + (rot * s).astype(F32), dtype)
    return np.concatenate([roped, x[..., rope_n:]], axis=-1).astype(F32)


def log_mass(w: np.ndarray) -> np.ndarray:
    """float32 ``log(max(w, 1))`` (correctly rounded from float64)."""
    return np.log(np.maximum(np.asarray(w, np.float64), 1.0)).astype(F32)


def pack_mid(level_k, level_v, level_w, plan, alpha_k_raw, alpha_v, alpha_pos, alpha_valid, alpha_count,
             recent_k, recent_v, recent_count, k_new, v_new, cos, sin, rope_n, dim, dtype, cos_dtype):
    """Packed K/V ``[B,G,length,dim]`` with the mass/mask coordinate (log_kv_pack.py:27-72).

    length = plan width + alpha_count + recent_count + new tokens.  K column
    ``kd`` holds log(max(w,1)) for valid pooled slots, 0 for exact/recent/new
    rows (-0.0 for valid exact rows: ``(~valid) * -10000``) and -10000 for
    invalid slots, cast to the storage dtype; invalid rows'
    K and V are zero.
    """
    idx, anchors, valid = plan
    B, G = idx.shape[:2]
    kd, vd = level_k.shape[-1], level_v.shape[-1]
    width = idx.shape[-1]
    T = k_new.shape[2]
    length = width + alpha_count + recent_count + T
    ka = np.zeros((B, G, length, dim), F32)
    va = np.zeros((B, G, length, dim), F32)
    cast = (lambda a: round_bf16(a)) if dtype == "bf16" else (lambda a: np.asarray(a, F32))
    if width:
        flat_k = np.asarray(level_k, F32).reshape(B, G, -1, kd)
        flat_v = np.asarray(level_v, F32).reshape(B, G, -1, vd)
        rows_k = np.take_along_axis(flat_k, idx[..., None], axis=2)
        rows_v = np.take_along_axis(flat_v, idx[..., None], axis=2)
        keys = rope_rows(rows_k, anchors, cos, sin, rope_n, dtype, cos_dtype)
        ka[:, :, :width, :kd] = np.where(valid[..., None], keys, 0)
        va[:, :, :width, :vd] = np.where(valid[..., None], rows_v, 0)
        weights = np.take_along_axis(np.asarray(level_w, F32).reshape(B, G, -1), idx, axis=2)
        ka[:, :, :width, kd] = cast(np.where(valid, log_mass(weights), F32(-10000.0)))
    at = width
    if alpha_count:
        ve = np.broadcast_to(np.asarray(alpha_valid, bool)[:, None, :alpha_count], (B, G, alpha_count))
        pe = np.broadcast_to(np.asarray(alpha_pos, np.int64)[:, None, :alpha_count], (B, G, alpha_count))
        keys = rope_rows(np.asarray(alpha_k_raw, F32)[:, :, :alpha_count], pe, cos, sin, rope_n, dtype, cos_dtype)
        ka[:, :, at:at + alpha_count, :kd] = np.where(ve[..., None], keys, 0)
        va[:, :, at:at + alpha_count, :vd] = np.where(ve[..., None], np.asarray(alpha_v, F32)[:, :, :alpha_count], 0)
        ka[:, :, at:at + alpha_count, kd] = cast(np.where(ve, F32(-0.0), F32(-10000.0)))  # (~valid) * -10000
        at += alpha_count
    ka[:, :, at:at + recent_count, :kd] = np.asarray(recent_k, F32)[:, :, :recent_count]
    va[:, :, at:at + recent_count, :vd] = np.asarray(recent_v, F32)[:, :, :recent_count]
    at += recent_count
    ka[:, :, at:at + T, :kd] = np.asarray(k_new, F32)
    va[:, :, at:at + T, :vd] = np.asarray(v_new, F32)
    return ka, va


def query_extra(scale: float, dtype: str) -> float:
    """The query's mass coordinate ``1/scale`` as stored in the query dtype (log_kv_cache.py:6459-6460)."""
    return float(round_bf16(np.asarray([1.0 / scale], F32))[0]) if dtype == "bf16" else float(F32(1.0 / scale))


def slot_attention(q, ka, va, scale: float, causal_tail: int, vd: int, dtype: str):
    """softmax(scale * [q, 1/scale] . K_aug) V with a lower-right causal tail, in float64.

    q [B, H, T, kd] (storage-dtype values); ka/va from ``pack_mid``.  Query head
    h reads KV group h // (H // G).  Returns [B, H, T, vd] float64.
    """
    q = np.asarray(q, np.float64)
    B, H, T, kd = q.shape
    G, S = ka.shape[1], ka.shape[2]
    rf = H // G
    qa = np.zeros((B, H, T, ka.shape[-1]), np.float64)
    qa[..., :kd] = q
    qa[..., kd] = query_extra(scale, dtype)
    kg = np.repeat(np.asarray(ka, np.float64), rf, axis=1)
    vg = np.repeat(np.asarray(va, np.float64)[..., :vd], rf, axis=1)
    scores = scale * np.einsum("bhtd,bhsd->bhts", qa, kg)
    if causal_tail:
        t = np.arange(T)[:, None]
        s = np.arange(S)[None, :]
        blocked = s > (S - T) + t
        scores = np.where(blocked[None, None], -np.inf, scores)
    m = scores.max(axis=-1, keepdims=True)
    p = np.exp(scores - m)
    p /= p.sum(axis=-1, keepdims=True)
    return np.einsum("bhts,bhsd->bhtd", p, vg)
