"""Unified (Ward / radius) route operators, restated in numpy (test infrastructure only).

Follows the reference's Torch reducer ``_UnifiedReduceTorch`` (litgpt/log_kv_cache.py:448-638)
with its helpers ``_unified_pack`` / ``_unified_pair_cost`` (:428-446), and the fused pair
distances / mirror of ``log_kv_route_triton.py:546-607``.  Every operation is float32 and
rounded as the reference writes it (one rounding per product, quotient, sum); the one sum over
features (the exact squared distance of a candidate pair, ``(diff * diff).sum(-1)`` in the
reference, whose order torch leaves to its vectorised CPU kernel) runs left to right here, and
the CUDA operators use the same order.

Flush level (``_semantic_route_unified``, log_kv_cache.py:3589-3688): ``pair_matrix``
(``_semantic_unified_pair_matrix`` :3185-3221, its two forms), ``reduce_lanes``
(``_semantic_unified_reduce_device`` :3246-3299 with the host loop of
``_semantic_unified_reduce_incremental`` :3301-3376), ``labels_batch``
(``_semantic_unified_labels_batch`` :3544-3568), ``route_tile`` (``_semantic_unified_tile``
:3578-3587) and ``ward_entry_index`` (``_semantic_ward_entry_index`` :2450-2474).  The Gram
products (one fused multiply-add per feature) and the exact-difference sums of the pair matrix run
left to right over the features (the reference leaves that order to its BLAS / vectorised CPU
kernels).
"""
from __future__ import annotations

import numpy as np

F32 = np.float32
INF_KEY = np.int64(0x7F800000) << np.int64(32)


def pair_distances(gram: np.ndarray, norm: np.ndarray) -> np.ndarray:
    """max((n_i + n_j) - 2 G_ij, 0) from the upper triangle of G, mirrored (route:556-607)."""
    gram = np.asarray(gram, F32)
    norm = np.asarray(norm, F32)
    L, M, _ = gram.shape
    d = np.maximum((norm[:, :, None] + norm[:, None, :]).astype(F32) - (F32(2) * gram).astype(F32), F32(0))
    upper = np.triu(np.ones((M, M), bool))
    return np.where(upper[None], d, np.transpose(d, (0, 2, 1))).astype(F32)


def mirror(dist: np.ndarray) -> np.ndarray:
    """Copy the upper triangle onto the lower one (route:546-553)."""
    M = dist.shape[1]
    upper = np.triu(np.ones((M, M), bool))
    return np.where(upper[None], dist, np.transpose(dist, (0, 2, 1))).astype(F32)


def pack(cost: np.ndarray, key: np.ndarray) -> np.ndarray:
    """(cost bits << 32) | key with -0.0 written as +0.0 (log_kv_cache.py:431-434)."""
    cost = np.where(cost == 0, F32(0), np.asarray(cost, F32)).astype(F32)
    return (cost.view(np.int32).astype(np.int64) << np.int64(32)) | np.asarray(key, np.int64)


def pair_cost(d2, mi, mj, ri, rj, limit, valid):
    """Ward cost and validity (log_kv_cache.py:437-445), float32 in the reference's order."""
    d2, mi, mj = np.asarray(d2, F32), np.asarray(mi, F32), np.asarray(mj, F32)
    denom = np.maximum((mi + mj).astype(F32), F32(1))
    valid = valid & (mi > 0) & (mj > 0)
    if limit is not None:
        distance = np.sqrt(d2).astype(F32)
        b1 = (np.asarray(ri, F32) + ((mj / denom).astype(F32) * distance).astype(F32)).astype(F32)
        b2 = (np.asarray(rj, F32) + ((mi / denom).astype(F32) * distance).astype(F32)).astype(F32)
        valid = valid & (np.maximum(b1, b2) <= limit)
    cost = (d2 * ((mi * mj).astype(F32) / denom).astype(F32)).astype(F32)
    return np.where(valid, cost, F32(np.inf)).astype(F32), valid


def sq_dist(x: np.ndarray, y: np.ndarray) -> F32:
    """sum_d (x_d - y_d)^2, left to right in float32."""
    acc = F32(0)
    for a, b in zip(x.tolist(), y.tolist()):
        d = F32(F32(a) - F32(b))
        acc = F32(acc + F32(d * d))
    return acc


class UnifiedReduce:
    """Mutual-nearest Ward rounds on [L, M] clusters (single-pass rounds).

    dist [L, M, M] squared centre distances (symmetric), mu [L, M, D] centres, mass [L, M],
    count [L] live clusters (rows < count), limits [L] radius limits or None, target clusters
    per lane.  ``step()`` runs one round and returns the lanes still active; ``finish()`` returns
    (per-lane merge traces [(left, right), ...] in round then (cost, left) order, alive [L, M],
    stuck [L]).  Arrays are updated in place.
    """

    def __init__(self, dist, mu, mass, count, limits, target, passes=1):
        self.passes = max(1, int(passes))
        self.dist = np.array(dist, F32)
        self.mu = np.array(mu, F32)
        self.mass = np.array(mass, F32)
        self.limits = None if limits is None else np.array(limits, F32)
        self.target = int(target)
        L, M = self.mass.shape
        self.L, self.M = L, M
        self.ids = np.arange(M, dtype=np.int64)
        self.count = np.array(count, np.int64).copy()
        self.alive = self.ids[None, :] < self.count[:, None]
        self.radius = np.zeros((L, M), F32)
        self.stuck = np.zeros(L, bool)
        self.traces = [[] for _ in range(L)]
        self.packed = np.full((L, M), INF_KEY, np.int64)
        for lane in range(L):
            for row in np.flatnonzero(self.alive[lane]):
                self.packed[lane, row] = self._scan(lane, row)

    def _scan(self, lane, row, excluded=None):
        lim = None if self.limits is None else self.limits[lane]
        mass = self.mass[lane] if excluded is None else np.where(excluded, F32(0), self.mass[lane]).astype(F32)
        cost, _ = pair_cost(self.dist[lane, row], self.mass[lane, row], mass, self.radius[lane, row],
                            self.radius[lane], lim, self.ids != row)
        return pack(cost, np.int64(row) ^ self.ids).min()

    def _sweeps(self, lane, valid, best, pair_c):
        """Frozen-centre sweeps of one lane (``_UnifiedReduceTorch._sweeps``, :564-588)."""
        M, ids = self.M, self.ids
        alive = self.alive[lane]
        matched = np.zeros(M, bool)
        rows = np.flatnonzero(valid)
        matched[rows] = True
        matched[best[rows]] = True
        restricted = self.packed[lane].copy()
        mate, extra = best.copy(), 0
        for _ in range(self.passes - 1):
            partner = np.clip((restricted & np.int64(0xFFFFFFFF)) ^ ids, 0, M - 1)
            for row in np.flatnonzero(alive & ~matched & matched[partner]):
                restricted[row] = self._scan(lane, row, excluded=matched)
            partner = np.clip((restricted & np.int64(0xFFFFFFFF)) ^ ids, 0, M - 1)
            cost = (restricted >> np.int64(32)).astype(np.int32).view(np.float32)
            more = (alive & ~matched & (ids < partner) & (partner[partner] == ids) & (cost < np.inf)
                    & ~matched[partner])
            extra += int(more.sum())
            rows = np.flatnonzero(more)
            matched[rows] = True
            matched[partner[rows]] = True
            mate = np.where(more, partner, mate)
            pair_c = np.where(more, cost, pair_c).astype(F32)
        return mate, pair_c, extra

    def step(self):
        M, ids = self.M, self.ids
        active = np.zeros(self.L, bool)
        for lane in range(self.L):
            packed = self.packed[lane]
            best = np.clip((packed & np.int64(0xFFFFFFFF)) ^ ids, 0, M - 1)
            cost = (packed >> np.int64(32)).astype(np.int32).view(np.float32)
            valid = self.alive[lane] & (ids < best) & (best[best] == ids) & (cost < np.inf)
            nprop = int(valid.sum())
            rejected = np.zeros(M, bool)
            bound = None
            if self.limits is not None:
                bound = np.zeros(M, F32)
                for row in np.flatnonzero(valid):
                    other = best[row]
                    exact2 = sq_dist(self.mu[lane, row], self.mu[lane, other])
                    exact = F32(np.sqrt(exact2))
                    ma, mb = self.mass[lane, row], self.mass[lane, other]
                    denom = max(F32(ma + mb), F32(1))
                    v1 = F32(self.radius[lane, row] + F32(F32(mb / denom) * exact))
                    v2 = F32(self.radius[lane, other] + F32(F32(ma / denom) * exact))
                    verified = max(v1, v2)
                    if verified > self.limits[lane]:
                        self.dist[lane, row, other] = exact2
                        self.dist[lane, other, row] = exact2
                        rejected[row] = rejected[other] = True
                        valid[row] = False
                    bound[row] = verified
            pair_c = np.where(valid, cost, F32(np.inf)).astype(F32)
            mate = best
            if self.passes > 1:
                mate, pair_c, extra = self._sweeps(lane, valid, best, pair_c)
                nprop += extra
            order = np.argsort(pair_c, kind="stable")[:M // 2]
            ok = pair_c[order] < np.inf
            ok &= np.cumsum(ok) <= (self.count[lane] - self.target)
            a = order[ok]
            b = mate[a]
            keep = np.zeros(M, bool)
            merged = np.zeros(M, bool)
            if len(a):
                self._merge(lane, a, b, bound, keep, merged)
            dirty = self.alive[lane] & ~keep & (merged[best] | rejected)
            for row in np.flatnonzero(dirty):
                self.packed[lane, row] = self._scan(lane, row)
            self.count[lane] -= int(ok.sum())
            remaining = self.count[lane] > self.target
            self.stuck[lane] |= remaining and nprop == 0
            active[lane] = remaining and nprop > 0
        return active

    def _merge(self, lane, a, b, bound, keep, merged):
        M, ids = self.M, self.ids
        dist, mass = self.dist[lane], self.mass[lane]
        ma, mb = mass[a].copy(), mass[b].copy()
        dab = dist[a, b].copy()
        total = (ma + mb).astype(F32)
        alpha = (ma / total).astype(F32)
        beta = (mb / total).astype(F32)
        shift = ((alpha * beta).astype(F32) * dab).astype(F32)
        keep[a] = True
        merged[a] = True
        merged[b] = True
        partner = np.zeros(M, np.int64)
        partner[a] = b
        pma, pmb, pdab = np.ones(M, F32), np.zeros(M, F32), np.zeros(M, F32)
        pma[a], pmb[a], pdab[a] = ma, mb, dab
        x_aa, x_ba = dist[a].copy(), dist[b].copy()                  # [n, M], read before any write
        x_ab, x_bb = dist[a[:, None], partner[None, :]].copy(), dist[b[:, None], partner[None, :]].copy()
        mass[a] = total
        mass[b] = 0
        self.alive[lane, b] = False
        if bound is not None:
            self.radius[lane, a] = bound[a]
        mu = self.mu[lane]
        mu[a] = (((ma[:, None] * mu[a]).astype(F32) + (mb[:, None] * mu[b]).astype(F32)).astype(F32)
                 / np.maximum(total, F32(1))[:, None]).astype(F32)
        al, be, sh = alpha[:, None], beta[:, None], shift[:, None]
        new = ((((al * x_aa).astype(F32) + (be * x_ba).astype(F32)).astype(F32)) - sh).astype(F32)
        is_keep = keep[None, :]
        qa, qb, qd = pma[None, :], pmb[None, :], pdab[None, :]
        qsum = (qa + qb).astype(F32)
        qal, qbe = (qa / qsum).astype(F32), (qb / qsum).astype(F32)
        qsh = ((qal * qbe).astype(F32) * qd).astype(F32)
        inner = ((((al * x_ab).astype(F32) + (be * x_bb).astype(F32)).astype(F32)) - sh).astype(F32)
        own_first = (((qal * new).astype(F32) + (qbe * inner).astype(F32)).astype(F32) - qsh).astype(F32)
        t1 = ((((qal * x_aa).astype(F32) + (qbe * x_ab).astype(F32)).astype(F32)) - qsh).astype(F32)
        t2 = ((((qal * x_ba).astype(F32) + (qbe * x_bb).astype(F32)).astype(F32)) - qsh).astype(F32)
        other_first = ((((al * t1).astype(F32) + (be * t2).astype(F32)).astype(F32)) - sh).astype(F32)
        both = np.where(a[:, None] < ids[None, :], own_first, other_first)
        new = np.maximum(np.where(is_keep, both, new), F32(0)).astype(F32)
        new[np.arange(len(a)), a] = 0
        alive = self.alive[lane]
        for m in range(len(a)):
            cols = np.flatnonzero(alive & ~keep)
            dist[cols, a[m]] = new[m, cols]
        for m in range(len(a)):
            cols = np.flatnonzero(alive)
            dist[a[m], cols] = new[m, cols]
        lim = None if self.limits is None else self.limits[lane]
        cost, valid = pair_cost(new, total[:, None], mass[None, :], self.radius[lane, a][:, None],
                                self.radius[lane][None, :], lim, alive[None, :] & (ids[None, :] != a[:, None]))
        packed_new = pack(cost, ids[None, :] ^ a[:, None])
        for m in range(len(a)):
            cols = np.flatnonzero(valid[m] & ~keep)
            self.packed[lane, cols] = np.minimum(self.packed[lane, cols], packed_new[m, cols])
        for m in range(len(a)):
            self.packed[lane, a[m]] = packed_new[m].min()
            self.traces[lane].append((int(a[m]), int(b[m])))

    def finish(self):
        traces = [np.asarray(t, np.int64).reshape(-1, 2) for t in self.traces]
        return traces, self.alive.copy(), self.stuck.copy()


# ------------------------------------------------------------------------------ flush level
ROUTE_TILE_BYTES = 64 << 20   # the CPU reference's distance budget per lane tile (log_kv_cache.py:3575)


def route_tile(lanes: int, tokens: int, budget: int = ROUTE_TILE_BYTES) -> int:
    """Lanes per tile: the largest balanced tile whose [M, M] float32 matrices fit `budget`
    (``_semantic_unified_tile``, log_kv_cache.py:3578-3587)."""
    widest = max(1, budget // max(1, 4 * tokens * tokens))
    tiles = -(-lanes // widest)
    return max(1, -(-lanes // max(tiles, 1)))


def _lr_sum(terms) -> np.ndarray:
    """Left-to-right float32 sum over the last axis (one rounding per addition)."""
    acc = np.zeros(terms.shape[:-1], F32)
    for d in range(terms.shape[-1]):
        acc = (acc + terms[..., d]).astype(F32)
    return acc


def fma32(a, b, c) -> np.ndarray:
    """float32 fused multiply-add a * b + c with one rounding (as CUDA's fmaf): the product and
    the sum are exact in float64 up to the sum's rounding, whose error TwoSum recovers; only a
    float64 sum lying exactly on a float32 midpoint with a nonzero error rounds differently, and is
    nudged one float64 ulp toward the error first."""
    p = np.asarray(a, np.float64) * np.asarray(b, np.float64)
    cc = np.asarray(c, np.float64)
    s = p + cc
    bb = s - p
    e = (p - (s - bb)) + (cc - bb)
    low = s.view(np.uint64) & np.uint64((1 << 29) - 1)
    fix = (low == np.uint64(1 << 28)) & (e != 0)
    if fix.any():
        s = np.where(fix, np.nextafter(s, np.where(e > 0, np.inf, -np.inf)), s)
    return s.astype(F32)


def pair_matrix(mu: np.ndarray) -> np.ndarray:
    """Squared centre distances [L, M, M] (``_semantic_unified_pair_matrix``, :3185-3221).

    M <= 32: exact differences, ``cdist(...).square()`` (the root rounded, then squared).
    Otherwise centred on each lane's first row: norm n_i = sum_d c_id^2, Gram G_ij = sum_d
    c_id c_jd (a fused multiply-add per feature, in order), d_ij = max((n_i + n_j) - 2 G_ij, 0),
    upper triangle mirrored.
    """
    mu = np.asarray(mu, F32)
    L, M, D = mu.shape
    if M <= 32:
        acc = np.zeros((L, M, M), F32)
        for d in range(D):
            diff = (mu[:, :, None, d] - mu[:, None, :, d]).astype(F32)
            acc = (acc + (diff * diff).astype(F32)).astype(F32)
        root = np.sqrt(acc).astype(F32)
        return mirror((root * root).astype(F32))
    c = (mu - mu[:, :1]).astype(F32)
    norm = _lr_sum((c * c).astype(F32))
    gram = np.zeros((L, M, M), F32)
    for d in range(D):
        gram = fma32(c[:, :, None, d], c[:, None, :, d], gram)
    return pair_distances(gram, norm)


def reduce_lanes(mu, counts, weights, *, target, radius_limits=None, strict=False, passes=1):
    """Mutual-nearest Ward rounds on a padded float32 [L, M, D] buffer, updated in place
    (``_semantic_unified_reduce_device`` :3246-3299 and the round loop of
    ``_semantic_unified_reduce_incremental`` :3301-3376).  Returns per-lane surviving rows
    (ascending) and merge pairs (left, right) in round, then (cost, left) order."""
    lanes = len(counts)
    active = [i for i, n in enumerate(counts) if n > target]
    survivors = [np.arange(n, dtype=np.int64) for n in counts]
    traces = [np.empty((0, 2), np.int64) for _ in counts]
    if not active:
        return survivors, traces
    if len(active) < lanes:
        size = max(counts[i] for i in active)
    else:
        size = mu.shape[1]
    sub = np.array(mu[active, :size], F32)
    w = np.asarray(weights, F32)[active, :size]
    limits = None if radius_limits is None else np.asarray([radius_limits[i] for i in active], F32)
    # Frozen-centre sweeps only for the uncapped global pass (radius limits keep one sweep).
    red = UnifiedReduce(pair_matrix(sub), sub, w, [counts[i] for i in active], limits, target,
                        passes if radius_limits is None else 1)
    last_round = 2 * size + 7
    for _ in range(last_round):
        if not red.step().any():
            break
    lane_traces, alive, stuck = red.finish()
    if strict and stuck.any():
        raise RuntimeError("unified routing has no finite merge cost to satisfy the cluster budget")
    mu[active, :size] = red.mu
    for j, i in enumerate(active):
        survivors[i] = np.flatnonzero(alive[j]).astype(np.int64)
        traces[i] = lane_traces[j]
    return survivors, traces


def labels_batch(sizes, survivors, traces):
    """Leaf -> compact surviving row, by pointer jumping over the merge forest
    (``_semantic_unified_labels_batch``, :3544-3568)."""
    sizes = np.asarray(sizes, np.int64)
    offsets = np.cumsum(sizes) - sizes
    parent = np.arange(int(sizes.sum()), dtype=np.int64)
    pairs = [np.asarray(t, np.int64) + off for t, off in zip(traces, offsets.tolist()) if len(t)]
    if pairs:
        pairs = np.concatenate(pairs)
        parent[pairs[:, 1]] = pairs[:, 0]
        while True:
            grand = parent[parent]
            if np.array_equal(parent, grand):
                break
            parent = grand
    compact = np.empty(len(parent), np.int64)
    compact[np.concatenate([np.asarray(r, np.int64) + off for r, off in zip(survivors, offsets.tolist())])] = \
        np.concatenate([np.arange(len(r), dtype=np.int64) for r in survivors])
    return np.split(compact[parent], offsets[1:])


def ward_entry_index(order, lo, has_mass, split):
    """Merged entry order of one Ward merge (``_semantic_ward_entry_index``, :2450-2474, for one
    keep side [0, split) and free side [split, n)): each side stably sorted by level order; an
    entry's key is the p_lo of the next entry with mass at or after it on its side (else its
    own order); the sides merge by their running maxima of that key, keep side first on ties."""
    order = np.asarray(order, np.int64)
    lo = np.asarray(lo, np.int64)
    has_mass = np.asarray(has_mass, bool)
    n = len(order)
    segment = (np.arange(n) >= split).astype(np.int64)
    perm = np.argsort((segment << 32) + order, kind="stable")
    o, l, h = order[perm], lo[perm], has_mass[perm]
    seg_end = np.where(segment == 0, split, n)
    ids = np.arange(n)
    following = np.minimum.accumulate(np.where(h, ids, n)[::-1])[::-1]
    effective = np.where(following < seg_end, l[np.minimum(following, n - 1)], o)
    running = np.maximum.accumulate((segment << 32) + effective) - (segment << 32)
    merge = np.argsort(running, kind="stable")
    return perm[merge]
