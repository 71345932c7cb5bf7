"""Per-lane log-structured ladder append (TEST INFRASTRUCTURE ONLY).

Restates, one (batch, group, cluster) lane at a time, what the reference does
for many lanes at once in
``LogStructuredKVCache._semantic_append_entries_batched``
(litgpt/log_kv_cache.py:1756-1929) with the merges of ``compact``
(:5217-5387, anchors via log_kv_position.merge_anchors :13-30), Beta's
``select_cuts``/``apply_cuts`` (litgpt/beta_log_kv.py:7-92) and the saturated
top-level fold ``_semantic_append_top_level_overflow_batched`` (:1670-1728).

Per level with ``c`` stored entries and ``m`` incoming rows the reference's
index plan is equivalent to: pool = stored[0:c] ++ cast(incoming), length c+m.
If c+m <= B' the incoming rows fill slots c..c+m-1.  Otherwise the first
2*ceil((c+m-B')/2) pool rows merge pairwise (or in Beta groups of four) into the
carry for the next level, the remaining pool rows become slots 0..n-1 and slots
n..B'-1 are zeroed.  On the top level the pool is folded left instead.
"""
from __future__ import annotations

from dataclasses import dataclass

import numpy as np

from .numerics import F32, dsum, seq_sum, to_storage

I64MAX = np.iinfo(np.int64).max
I64MIN = np.iinfo(np.int64).min


@dataclass
class Rows:
    """A block of ladder entries (the 8 first-order fields the flush touches)."""
    k: np.ndarray      # [n, Dk] float32 (storage-rounded, or float32 carry)
    v: np.ndarray      # [n, Dv] float32
    w: np.ndarray      # [n] float32
    lo: np.ndarray     # [n] int64
    hi: np.ndarray     # [n] int64
    swp: np.ndarray    # [n] int64
    order: np.ndarray  # [n] int64
    pad: np.ndarray    # [n] bool

    def __len__(self) -> int:
        return int(self.w.shape[0])

    def take(self, idx) -> "Rows":
        return Rows(self.k[idx], self.v[idx], self.w[idx], self.lo[idx], self.hi[idx],
                    self.swp[idx], self.order[idx], self.pad[idx])

    def cast(self, dtype: str) -> "Rows":
        return Rows(to_storage(self.k, dtype), to_storage(self.v, dtype), self.w.astype(np.float32),
                    self.lo.astype(np.int64), self.hi.astype(np.int64), self.swp.astype(np.int64),
                    self.order.astype(np.int64), self.pad.astype(bool))

    @staticmethod
    def cat(a: "Rows", b: "Rows") -> "Rows":
        return Rows(*(np.concatenate([x, y], axis=0) for x, y in zip(a.fields(), b.fields())))

    def fields(self):
        return (self.k, self.v, self.w, self.lo, self.hi, self.swp, self.order, self.pad)

    @staticmethod
    def empty(dk: int, dv: int) -> "Rows":
        return Rows(np.zeros((0, dk), F32), np.zeros((0, dv), F32), np.zeros(0, F32),
                    np.zeros(0, np.int64), np.zeros(0, np.int64), np.zeros(0, np.int64),
                    np.zeros(0, np.int64), np.zeros(0, bool))

    @staticmethod
    def tokens(k, v, pos, order) -> "Rows":
        """Exact token rows: w=1, p_lo=p_hi=sum_wp=position (log_kv_cache.py:4294-4304)."""
        pos = np.asarray(pos, dtype=np.int64)
        n = pos.shape[0]
        return Rows(np.asarray(k, F32), np.asarray(v, F32), np.ones(n, F32), pos.copy(), pos.copy(), pos.copy(),
                    np.asarray(order, dtype=np.int64), np.zeros(n, bool))


def merge_pairs(rows: Rows) -> Rows:
    """Rows (2i, 2i+1) -> entry i: count-weighted mean in float32 without FMA.

    alpha = wa / max(wa+wb, 1e-8); k = alpha*ka + (1-alpha)*kb (compact,
    log_kv_cache.py:5296-5306); p_lo/p_hi over positive-weight sides
    (merge_anchors), sum_wp added, order = min, pad = AND (:1561-1568).
    """
    a, b = rows.take(slice(0, None, 2)), rows.take(slice(1, None, 2))
    total = (a.w + b.w).astype(F32)
    alpha = (a.w / np.maximum(total, F32(1e-8))).astype(F32)
    beta = (F32(1.0) - alpha).astype(F32)
    k = ((alpha[:, None] * a.k).astype(F32) + (beta[:, None] * b.k).astype(F32)).astype(F32)
    v = ((alpha[:, None] * a.v).astype(F32) + (beta[:, None] * b.v).astype(F32)).astype(F32)
    ra, rb = a.w > 0, b.w > 0
    lo = np.where(ra & rb, np.minimum(a.lo, b.lo), np.where(ra, a.lo, b.lo))
    hi = np.where(ra & rb, np.maximum(a.hi, b.hi), np.where(ra, a.hi, b.hi))
    return Rows(k, v, total, lo, hi, a.swp + b.swp, np.minimum(a.order, b.order), a.pad & b.pad)


def beta_layout(lengths) -> np.ndarray:
    """Groups of four per lane, never across lanes: rows (start, width, dst).

    Follows make_layout (litgpt/beta_log_kv.py:7-18): widths are 4 except a
    final 2 for a lane length that is 2 mod 4; dst = start // 2.
    """
    out = []
    base = 0
    for n in lengths:
        n = int(n)
        if n < 0 or n % 2:
            raise ValueError("Beta compaction requires even nonnegative lane lengths")
        for off in range(0, n, 4):
            start = base + off
            out.append((start, min(4, n - off), start // 2))
        base += n
    return np.asarray(out, dtype=np.int64).reshape(-1, 3)


def beta_cost_cut(g: Rows, width: int) -> tuple[int, np.ndarray]:
    """Cut of one group: argmin over cuts (2, 1, 3) of the normalised weighted SSE.

    select_cuts (beta_log_kv.py:29-46): ties keep the earlier candidate, so
    2|2 wins a tie, then 1|3; a width-2 group always reports the sentinel 1.
    Returns (cut, costs[3]).
    """
    offs = np.arange(4)
    valid = offs < width
    w = np.zeros(4, F32)
    w[:width] = g.w[:width]
    total = max(seq_sum(w[:, None])[0], F32(1e-12))
    costs = np.zeros(3, F32)
    for x_rows in (g.k, g.v):
        x = np.zeros((4, x_rows.shape[1]), F32)
        x[:width] = x_rows[:width]
        energy = max(F32(seq_sum((dsum(x * x) * w)[:, None])[0] / total), F32(1e-12))
        for j, cut in enumerate((2, 1, 3)):
            left = valid & (offs < cut)
            for mask in (left, valid & ~left):
                weights = (w * mask).astype(F32)
                mean = (seq_sum(x * weights[:, None]) / max(seq_sum(weights[:, None])[0], F32(1e-12))).astype(F32)
                loss = seq_sum((dsum((x - mean[None, :]) ** 2) * weights)[:, None])[0]
                costs[j] = F32(costs[j] + F32(loss / energy))
    if width == 2:
        return 1, costs
    return (2, 1, 3)[int(np.argmin(costs))], costs


def beta_apply(g: Rows, width: int, cut: int) -> Rows:
    """Two mass-weighted entries (one for a width-2 tail) from a recorded cut.

    apply_cuts (beta_log_kv.py:49-92): sums over the group run in row order,
    K/V = sum(w*x) / max(mass, 1e-12); positions over positive-weight members.
    """
    offs = np.arange(4)
    valid = offs < width
    w = np.zeros(4, F32)
    w[:width] = g.w[:width]
    kx = np.zeros((4, g.k.shape[1]), F32)
    vx = np.zeros((4, g.v.shape[1]), F32)
    kx[:width], vx[:width] = g.k[:width], g.v[:width]
    meta = []
    for arr, fill in ((g.lo, 0), (g.hi, 0), (g.swp, 0), (g.order, 0)):
        z = np.full(4, fill, np.int64)
        z[:width] = arr[:width]
        meta.append(z)
    lo4, hi4, swp4, ord4 = meta
    pad4 = np.ones(4, bool)
    pad4[:width] = g.pad[:width]
    outs = []
    for side in (0, 1):
        if width == 2:
            mask = valid if side == 0 else np.zeros(4, bool)
        else:
            mask = valid & ((offs < cut) if side == 0 else (offs >= cut))
        if side == 1 and width != 4:
            break
        weights = (w * mask).astype(F32)
        mass = seq_sum(weights[:, None])[0]
        denom = max(mass, F32(1e-12))
        k = (seq_sum(kx * weights[:, None]) / denom).astype(F32)
        v = (seq_sum(vx * weights[:, None]) / denom).astype(F32)
        live = mask & (w > 0)
        lo = np.min(np.where(live, lo4, I64MAX)) if mass > 0 else 0
        hi = np.max(np.where(live, hi4, I64MIN)) if mass > 0 else 0
        swp = int(np.sum(np.where(mask, swp4, 0)))
        order = int(np.min(np.where(mask, ord4, I64MAX)))
        pad = bool(np.all(pad4 | ~mask))
        outs.append((k, v, mass, lo, hi, swp, order, pad))
    return Rows(np.stack([o[0] for o in outs]), np.stack([o[1] for o in outs]),
                np.asarray([o[2] for o in outs], F32), np.asarray([o[3] for o in outs], np.int64),
                np.asarray([o[4] for o in outs], np.int64), np.asarray([o[5] for o in outs], np.int64),
                np.asarray([o[6] for o in outs], np.int64), np.asarray([o[7] for o in outs], bool))


def _grouped(x: np.ndarray, n: int, fill=0):
    """Pad a per-row array of one lane to [ceil(n/4), 4, ...] groups."""
    ng = (n + 3) // 4
    out = np.full((ng * 4,) + x.shape[1:], fill, dtype=x.dtype)
    out[:n] = x[:n]
    return out.reshape((ng, 4) + x.shape[1:])


def beta_costs_all(rows: Rows) -> np.ndarray:
    """Costs [groups, 3] for cuts (2, 1, 3) of every group of one lane (vectorised beta_cost_cut)."""
    n = len(rows)
    w = _grouped(rows.w, n)                                   # [NG, 4]
    width = np.minimum(4, n - 4 * np.arange(w.shape[0]))
    valid = np.arange(4)[None, :] < width[:, None]
    total = np.maximum(seq_sum(w.T), F32(1e-12))             # [NG]
    costs = np.zeros((w.shape[0], 3), F32)
    offs = np.arange(4)[None, :]
    for xr in (rows.k, rows.v):
        x = _grouped(xr, n)                                   # [NG, 4, D]
        energy = np.maximum((seq_sum((dsum(x * x) * w).T) / total).astype(F32), F32(1e-12))
        for j, cut in enumerate((2, 1, 3)):
            left = valid & (offs < cut)
            for mask in (left, valid & ~left):
                om = (w * mask).astype(F32)                   # [NG, 4]
                den = np.maximum(seq_sum(om.T), F32(1e-12))   # [NG]
                mean = (seq_sum(np.moveaxis(x * om[..., None], 1, 0)) / den[:, None]).astype(F32)   # [NG, D]
                loss = seq_sum((dsum((x - mean[:, None, :]) ** 2) * om).T)                        # [NG]
                costs[:, j] = (costs[:, j] + (loss / energy).astype(F32)).astype(F32)
    return costs


def beta_merge(rows: Rows, cuts=None) -> tuple[Rows, np.ndarray]:
    """One lane's pair rows -> half as many entries via Beta groups (merge_blocks, :95-105).

    All groups are evaluated at once with the same left-to-right sums as
    ``beta_cost_cut`` / ``beta_apply``.
    """
    n = len(rows)
    if n == 0:
        return Rows.empty(rows.k.shape[1], rows.v.shape[1]), np.zeros(0, np.uint8)
    ng = (n + 3) // 4
    width = np.minimum(4, n - 4 * np.arange(ng))
    if cuts is None:
        costs = beta_costs_all(rows)
        chosen = np.asarray((2, 1, 3), np.uint8)[np.argmin(costs, axis=1)]
        chosen = np.where(width == 2, np.uint8(1), chosen).astype(np.uint8)
    else:
        chosen = np.asarray(cuts, np.uint8)
    w = _grouped(rows.w, n)
    k4, v4 = _grouped(rows.k, n), _grouped(rows.v, n)
    lo4, hi4 = _grouped(rows.lo, n), _grouped(rows.hi, n)
    swp4, ord4 = _grouped(rows.swp, n), _grouped(rows.order, n)
    pad4 = _grouped(rows.pad, n, fill=True)
    valid = np.arange(4)[None, :] < width[:, None]
    offs = np.arange(4)[None, :]
    cut = chosen.astype(np.int64)[:, None]
    sides = []
    for side in (0, 1):
        if side == 0:
            mask = np.where((width == 2)[:, None], valid, valid & (offs < cut))
        else:
            mask = np.where((width == 2)[:, None], False, valid & (offs >= cut))
        om = (w * mask).astype(F32)
        mass = seq_sum(om.T)
        den = np.maximum(mass, F32(1e-12))
        kk = (seq_sum(np.moveaxis(k4 * om[..., None], 1, 0)) / den[:, None]).astype(F32)
        vv = (seq_sum(np.moveaxis(v4 * om[..., None], 1, 0)) / den[:, None]).astype(F32)
        live = mask & (w > 0)
        lo = np.where(mass > 0, np.min(np.where(live, lo4, I64MAX), axis=1), 0)
        hi = np.where(mass > 0, np.max(np.where(live, hi4, I64MIN), axis=1), 0)
        swp = np.sum(np.where(mask, swp4, 0), axis=1)
        order = np.min(np.where(mask, ord4, I64MAX), axis=1)
        pad = np.all(pad4 | ~mask, axis=1)
        sides.append((kk, vv, mass, lo, hi, swp, order, pad))
    # Interleave left/right per group; width-2 groups emit only the left entry.
    keep_right = width == 4
    fields = []
    for f in range(8):
        left, right = sides[0][f], sides[1][f]
        inter = np.stack([left, right], axis=1).reshape((2 * ng,) + left.shape[1:])
        sel = np.stack([np.ones(ng, bool), keep_right], axis=1).reshape(-1)
        fields.append(inter[sel])
    return Rows(*fields), chosen


class Ladder:
    """The 8 ladder fields of every lane, in the reference's buffer layout.

    Arrays have shape [B, G, K, L, B'] (+ feature dim) exactly like
    level_k/level_v/level_w/level_p_lo/level_p_hi/level_sum_wp/level_order/
    pad_mask; ``count`` mirrors level_count.
    """

    def __init__(self, batch, groups, clusters, levels, slots, dk, dv, dtype):
        shape = (batch, groups, clusters, levels, slots)
        self.dtype = dtype
        self.L, self.Bs = levels, slots
        self.k = np.zeros(shape + (dk,), F32)
        self.v = np.zeros(shape + (dv,), F32)
        self.w = np.zeros(shape, F32)
        self.lo = np.full(shape, I64MAX, np.int64)
        self.hi = np.full(shape, -1, np.int64)
        self.swp = np.zeros(shape, np.int64)
        self.order = np.zeros(shape, np.int64)
        self.pad = np.zeros(shape, bool)
        self.count = np.zeros(shape[:4], np.int64)

    def arrays(self):
        return (self.k, self.v, self.w, self.lo, self.hi, self.swp, self.order, self.pad)

    def read(self, b, g, c, ell, sl) -> Rows:
        return Rows(*(x[b, g, c, ell, sl].copy() for x in self.arrays()))

    def write(self, b, g, c, ell, start, rows: Rows) -> None:
        n = len(rows)
        for dst, src in zip(self.arrays(), rows.cast(self.dtype).fields()):
            dst[b, g, c, ell, start:start + n] = src

    def zero(self, b, g, c, ell, sl) -> None:
        for x in self.arrays():
            x[b, g, c, ell, sl] = 0

    def clear_lane(self, b, g, c) -> None:
        """_semantic_clear_clusters (:2476-2516): every level field of the lane becomes 0."""
        for x in self.arrays():
            x[b, g, c] = 0
        self.count[b, g, c] = 0

    def entries(self, b, g, c) -> Rows:
        """Stored entries in ladder order (level 0 first, slots ascending)."""
        parts = [self.read(b, g, c, ell, slice(0, int(self.count[b, g, c, ell]))) for ell in range(self.L)]
        out = parts[0]
        for p in parts[1:]:
            out = Rows.cat(out, p)
        return out

    def top_fold(self, b, g, c, pool: Rows, rem: int) -> None:
        """Saturated top level: slot 0 = left fold of pool[0..rem], slots 1.. = pool[rem+1..].

        Each fold step is a pairwise merge rounded to the storage dtype, as the
        reference's per-step ``.to(field dtype)`` does (:1716-1722).
        """
        ell = self.L - 1
        acc = pool.take(slice(0, 1))
        for t in range(1, rem + 1):
            acc = merge_pairs(Rows.cat(acc, pool.take(slice(t, t + 1)))).cast(self.dtype)
        self.write(b, g, c, ell, 0, acc)
        self.write(b, g, c, ell, 1, pool.take(slice(rem + 1, rem + self.Bs)))
        self.count[b, g, c, ell] = self.Bs

    def append(self, b, g, c, stage: Rows, beta: bool, replay_cuts=None, cut_log=None) -> None:
        """Append ``stage`` rows to lane (b, g, c), cascading carries upward."""
        for ell in range(self.L):
            m = len(stage)
            if m == 0:
                return
            cnt = int(self.count[b, g, c, ell])
            if cnt + m <= self.Bs:
                self.write(b, g, c, ell, cnt, stage)
                self.count[b, g, c, ell] = cnt + m
                return
            pool = Rows.cat(self.read(b, g, c, ell, slice(0, cnt)), stage.cast(self.dtype))
            rem = cnt + m - self.Bs
            if ell == self.L - 1:
                self.top_fold(b, g, c, pool, rem)
                return
            npair = 2 * ((rem + 1) // 2)
            head = pool.take(slice(0, npair))
            if beta:
                cuts = None if replay_cuts is None else replay_cuts[ell]
                carry, chosen = beta_merge(head, cuts)
                if cut_log is not None:
                    cut_log.append((ell, chosen))
            else:
                carry = merge_pairs(head)
            surv = pool.take(slice(npair, None))
            self.write(b, g, c, ell, 0, surv)
            self.zero(b, g, c, ell, slice(len(surv), self.Bs))
            self.count[b, g, c, ell] = len(surv)
            stage = carry
