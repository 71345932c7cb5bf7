"""Attach-route decisions for archived tokens (TEST INFRASTRUCTURE ONLY).

Restates ``_semantic_attach_decide`` / ``_semantic_attach_plan_torch``
(litgpt/log_kv_cache.py:4597-4680) with the frozen-centroid cost of
``_semantic_existing_assignments`` (:2649-2681), which is also what the fused
``_attach_assign`` kernel evaluates when every cluster is alive
(litgpt/log_kv_route_triton.py:841-891).

For each (batch, group) lane and each valid token, in position order:
  semantic_c = max((|x|^2 + |mu_c|^2) - 2 x.mu_c, 0)
  cost_c     = semantic_c + eta * gap_c / (gap_c + g0),  gap_c = max(pos - p_hi_c, 0)
  winner     = first argmin of cost over live clusters
  direct     = some cluster live and semantic_winner <= lam * s_h
Orphans (not direct) first seed up to one new cluster per free slot by
farthest-point picks (the orphan with the largest semantic_winner, then the
orphan farthest from all picks so far), then join the nearest live-or-seeded
cluster by exact distance.  Feature-axis sums use the canonical order of
``numerics.dsum``.
"""
from __future__ import annotations

import numpy as np

from .numerics import F32, dsum, ddot

I64MAX = np.iinfo(np.int64).max


def position_order(host_pos: np.ndarray, counts) -> np.ndarray:
    """Stable argsort by position with padding (index >= count) last (:4603-4605)."""
    B, T = host_pos.shape
    valid = np.arange(T)[None, :] < np.asarray(counts)[:, None]
    return np.argsort(np.where(valid, host_pos, I64MAX), axis=1, kind="stable")


def frozen_costs(x, pos, mu, alive, p_hi, s_h, eta, g0, lam):
    """Per token: winner, semantic of winner, direct flag, plus the winner's margin.

    x [T, D] float32, pos [T] int64, mu [K, D], alive [K], p_hi [K], s_h scalar.
    """
    xx = dsum((x * x).astype(F32))                                   # [T]
    mm = dsum((mu * mu).astype(F32))                                 # [K]
    cross = ddot(x[:, None, :], mu[None, :, :])                      # [T, K]
    semantic = np.maximum(((xx[:, None] + mm[None, :]).astype(F32) - (F32(2) * cross)).astype(F32), F32(0))
    gap = np.maximum((pos[:, None] - p_hi[None, :]).astype(F32), F32(0))
    temporal = (F32(eta) * (gap / (gap + F32(g0))).astype(F32)).astype(F32)
    cost = (semantic + temporal).astype(F32)
    cost = np.where(alive[None, :], cost, np.inf).astype(F32)
    winner = np.argmin(cost, axis=1)
    s_winner = semantic[np.arange(len(x)), winner]
    direct = bool(alive.any()) & (s_winner <= F32(F32(lam) * F32(s_h)))
    return winner, s_winner, direct, cost


def decide_lane(x, pos, count, mu, alive, p_hi, s_h, eta, g0, lam, free_slots, n_seed):
    """Final cluster (int) per token of one lane, in position order.

    x: [T, D] rows already permuted into position order, pos likewise.
    free_slots: ascending non-live cluster ids of this lane; n_seed: the
    maximum number of free slots over all lanes of the flush (the reference
    runs that many picks everywhere and uses only the first min(free, orphans)).
    Returns (assign [T] int64, -1 past count; margins dict for near-tie logging).
    """
    T, K = x.shape[0], mu.shape[0]
    valid = np.arange(T) < count
    winner, s_winner, direct, cost = frozen_costs(x, pos, mu, alive, p_hi, s_h, eta, g0, lam)
    direct = direct & valid
    orphan = valid & ~direct
    assign = np.where(direct, winner, -1).astype(np.int64)
    mu_ext = np.concatenate([mu.astype(F32), np.zeros((1, mu.shape[1]), F32)])
    cand = np.concatenate([alive.astype(bool), [False]])
    picked, used = [], []
    if n_seed:
        sw = np.where(orphan, s_winner, -np.inf)
        nxt = int(np.argmax(sw))
        picked.append(nxt)
        dist = np.where(orphan, dsum(((x - x[nxt]) ** 2).astype(F32)), -np.inf)
        for _ in range(n_seed - 1):
            dist[nxt] = -np.inf
            nxt = int(np.argmax(dist))
            picked.append(nxt)
            dist = np.minimum(dist, dsum(((x - x[nxt]) ** 2).astype(F32)))
        n_use = min(len(free_slots), int(orphan.sum()))
        for i, t in enumerate(picked):
            use = i < n_use
            used.append(use)
            if use:
                mu_ext[free_slots[i]] = x[t]
                cand[free_slots[i]] = True
    dist = np.sqrt(dsum(((x[:, None, :] - mu_ext[None, :K, :]) ** 2).astype(F32))).astype(F32)
    dist = np.where(cand[None, :K], dist, np.inf)
    nearest = np.argmin(dist, axis=1)
    assign = np.where(orphan, nearest, assign)
    for i, t in enumerate(picked):
        if used[i]:
            assign[t] = free_slots[i]
    assign[~valid] = -1
    return assign, dict(cost=cost, dist=dist, s_winner=s_winner, direct=direct)


def attach_decide(x_rows, positions, host_pos, counts, centroid, alive, p_hi, s_h, eta, g0, lam):
    """Attach decisions for a whole flush: (assign [B, G, T] int8 in position order, order [B, T]).

    x_rows: archived keys [B, G, T, D] (storage values as float32) in archive order;
    positions/host_pos: [B, T] positions of the archive rows (0 for padding).
    """
    B, G, T, D = x_rows.shape
    K = centroid.shape[2]
    order = position_order(host_pos, counts)
    free = [[[c for c in range(K) if not alive[b, g, c]] for g in range(G)] for b in range(B)]
    n_seed = max(len(f) for row in free for f in row)
    assign = np.full((B, G, T), -1, np.int64)
    for b in range(B):
        perm = order[b]
        for g in range(G):
            a, _ = decide_lane(x_rows[b, g, perm].astype(F32), positions[b, perm], int(counts[b]),
                               centroid[b, g].astype(F32), alive[b, g].astype(bool), p_hi[b, g],
                               float(s_h[b, g]), eta, g0, lam, free[b][g], n_seed)
            assign[b, g] = a
    return assign.astype(np.int8), order


def attach_assign_kernel(x, positions, order, counts, centroid, alive, p_hi, s_h, eta, g0, lam):
    """Restatement of the fused ``attach_assign`` plugin (route_triton.py:894-917), all clusters live.

    x [B, G, T, D]; order [B, T] token offsets by position; counts [B].
    Returns int8 [B, G, T] with -1 past each row's count.  Orphans take the
    nearest live cluster by exact squared distance (no square root, no seeds).
    """
    B, G, T, D = x.shape
    out = np.full((B, G, T), -1, np.int8)
    for b in range(B):
        n = int(counts[b])
        offs = order[b, :n]
        for g in range(G):
            xs = x[b, g, offs].astype(F32)
            mu = centroid[b, g].astype(F32)
            live = alive[b, g].astype(bool)
            winner, _sw, direct, _ = frozen_costs(xs, positions[b, offs], mu, live, p_hi[b, g],
                                                  float(s_h[b, g]), eta, g0, lam)
            exact = dsum(((xs[:, None, :] - mu[None, :, :]) ** 2).astype(F32))
            nearest = np.argmin(np.where(live[None, :], exact, np.inf), axis=1)
            out[b, g, :n] = np.where(direct, winner, nearest).astype(np.int8)
    return out
