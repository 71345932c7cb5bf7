"""Whole flush of the in-scope SemanticLogKV configuration (TEST INFRASTRUCTURE ONLY).

``OracleCache`` mirrors the state of the reference's ``LogStructuredKVCache``
(litgpt/log_kv_cache.py:681-1133) for semantic clusters with K > 1, mid
anchors, the Alpha exact-span pool, optional Beta, no second-order stats and
no segments, and restates its commit path:

  add_recent             _semantic_add_recent :5668-5718
  flush of F tokens      _semantic_flush_tokens :5609-5666
  Alpha select/partition _alpha_route_flush :3903-4003
  attach decisions       _semantic_attach_decide :4597-4634 (oracle.attach)
  grouping / new slots   _semantic_attach_commit :4682-4707, _semantic_new_clusters :2268-2298
  ordinary joins         _semantic_commit_joins_unsegmented :4116-4175, _semantic_apply_join_plan :4225-4361
  late (delayed) joins   _alpha_commit_joins :3690-3788
  ladder append          oracle.ladder (== _semantic_append_entries_batched :1756-1929)
  unified route          _semantic_route_unified :3589-3688 (oracle.unified), Ward merges of old
                         clusters _semantic_ward_merge_batch :2517-2593

Storage-dtype values are float32 arrays holding exact bf16 values when the
cache dtype is bf16.
"""
from __future__ import annotations

import math

import numpy as np

from . import alpha as A
from .attach import attach_decide
from .ladder import Ladder, Rows
from . import unified as U
from .numerics import F32, seq_sum, to_storage


def ladder_geometry(batch, groups, max_seq, dk, dv, B, clusters, exact, element_size):
    """(B', L) after the Alpha byte budget (log_kv_cache.py:855-899)."""
    levels = max(2, math.ceil(math.log2(max_seq / max(clusters * B, 1) + 1.0)) + 2)
    if not exact:
        return B, levels
    packed_dim = ((max(dk + 1, dv) + 7) // 8) * 8
    entry_bytes = (dk + dv + 2 * packed_dim) * element_size + 41
    exact_bytes = exact * (groups * (dk + dv + 2 * packed_dim) * element_size + 9)
    baseline = groups * clusters * levels * (B * entry_bytes + 2)
    for cand in range(B - 1, 1, -1):
        lv = max(2, math.ceil(math.log2(max_seq / (clusters * cand) + 1.0)) + 2)
        needed = groups * clusters * lv * (cand * entry_bytes + 2) + exact_bytes
        if needed <= baseline:
            return cand, lv
    raise ValueError("compressed ladder budget is too small for alpha_exact_tokens")


class OracleCache:
    def __init__(self, *, batch, groups, max_seq, dim, B, recent, clusters, granularity, exact, span_cap,
                 beta, dtype="fp32", s_h=None, eta=1.0, g0=2048.0, lam=1.0, unified=False, merge_passes=1):
        self.batch, self.groups, self.dim, self.K = batch, groups, dim, clusters
        self.unified, self.merge_passes = bool(unified), int(merge_passes)
        self.dtype = dtype
        self.max_seq = max_seq
        self.recent_size, self.granularity = recent, granularity
        self.exact, self.span_cap, self.beta = exact, span_cap, beta
        self.eta, self.g0, self.lam = eta, g0, lam
        esize = 4 if dtype == "fp32" else 2
        self.B_prime, self.L = ladder_geometry(batch, groups, max_seq, dim, dim, B, clusters, exact, esize)
        cap = 2 * recent
        self.recent_capacity = cap
        self.recent_k = np.zeros((batch, groups, cap, dim), F32)
        self.recent_k_raw = np.zeros((batch, groups, cap, dim), F32)
        self.recent_v = np.zeros((batch, groups, cap, dim), F32)
        self.recent_pos = np.zeros((batch, cap), np.int64)
        self.recent_ends = np.zeros((batch, cap), bool)
        self.recent_count = 0
        self.token_count = 0
        self.alpha_k_raw = np.zeros((batch, groups, exact, dim), F32)
        self.alpha_v = np.zeros((batch, groups, exact, dim), F32)
        self.alpha_pos = np.zeros((batch, exact), np.int64)
        self.alpha_valid = np.zeros((batch, exact), bool)
        self.alpha_spans = [[] for _ in range(batch)]
        self.alpha_positions = [[] for _ in range(batch)]
        self.alpha_count = 0
        self.ladder = Ladder(batch, groups, clusters, self.L, self.B_prime, dim, dim, dtype)
        self.centroid = np.zeros((batch, groups, clusters, dim), F32)
        self.n_eff = np.zeros((batch, groups, clusters), F32)
        self.n_total = np.zeros((batch, groups, clusters), np.int64)
        self.p_hi_c = np.full((batch, groups, clusters), -1, np.int64)
        self.level0_phase = np.zeros((batch, groups, clusters), np.int64)
        self.alive = np.zeros((batch, groups, clusters), bool)
        sh = 1.0 if s_h is None else s_h
        self.s_h = np.broadcast_to(np.asarray(sh, F32), (batch, groups)).astype(F32)
        self.trace = []          # per flush: dict of decisions, for near-tie reporting

    # ------------------------------------------------------------------ window
    def add_recent(self, k, v, k_raw, positions, span_ends):
        """Append a chunk to the window; flush granularity-sized blocks on overflow."""
        n = k.shape[2]
        if n > self.recent_size:
            raise ValueError(f"chunk size {n} exceeds recent_size {self.recent_size}")
        if self.token_count + n > self.max_seq:
            raise RuntimeError("token overflow")
        self.token_count += n
        if self.recent_count + n > self.recent_capacity:
            raise RuntimeError("recent buffer overflow")
        dst = slice(self.recent_count, self.recent_count + n)
        self.recent_k[:, :, dst] = to_storage(k, self.dtype)
        self.recent_k_raw[:, :, dst] = to_storage(k_raw, self.dtype)
        self.recent_v[:, :, dst] = to_storage(v, self.dtype)
        self.recent_pos[:, dst] = positions
        self.recent_ends[:, dst] = span_ends
        self.recent_count += n
        overflow = self.recent_count - self.recent_size
        if overflow > 0:
            gran = self.granularity
            pending = gran * ((overflow + gran - 1) // gran)
            while pending > 0:
                take = min(gran, pending)
                if take > self.recent_count:
                    raise RuntimeError("cannot flush more tokens than the window holds")
                self.flush(take)
                remaining = self.recent_count - take
                for arr in (self.recent_k, self.recent_k_raw, self.recent_v):
                    arr[:, :, :remaining] = arr[:, :, take:self.recent_count].copy()
                    arr[:, :, remaining:self.recent_count] = 0
                for arr in (self.recent_pos, self.recent_ends):
                    arr[:, :remaining] = arr[:, take:self.recent_count].copy()
                    arr[:, remaining:self.recent_count] = 0
                self.recent_count = remaining
                pending -= take

    # ------------------------------------------------------------------ flush
    def flush(self, T):
        B, G, D, P = self.batch, self.groups, self.dim, self.exact
        k_raw = self.recent_k_raw[:, :, :T].copy()
        v = self.recent_v[:, :, :T].copy()
        positions = self.recent_pos[:, :T].copy()
        ends = self.recent_ends[:, :T].copy()
        W = self.alpha_count
        keys = np.concatenate([self.alpha_k_raw[:, :, :W], k_raw], axis=2)
        vals = np.concatenate([self.alpha_v[:, :, :W], v], axis=2)
        pos = np.concatenate([self.alpha_pos[:, :W], positions], axis=1)
        cut = A.cut_spans(self.alpha_spans, self.alpha_positions, positions.tolist(), ends.tolist(), W, self.span_cap)
        if cut is None:
            sel = A.Selection([[] for _ in range(B)], [[] for _ in range(B)], [[] for _ in range(B)],
                              [[] for _ in range(B)])
            scores = None
        else:
            scores = A.score_spans(keys, vals, cut, beta_novelty=self.beta, centroids=self.centroid,
                                   centroid_valid=self.alive)
            sel = A.choose_spans(cut, scores, P)
        # Pool rewrite (gather with zero fill) and archive rows.
        self.alpha_k_raw[:] = 0
        self.alpha_v[:] = 0
        self.alpha_pos[:] = 0
        self.alpha_valid[:] = False
        for b, keep in enumerate(sel.keep):
            n = len(keep)
            self.alpha_k_raw[b, :, :n] = keys[b][:, keep]
            self.alpha_v[b, :, :n] = vals[b][:, keep]
            self.alpha_pos[b, :n] = pos[b, keep]
            self.alpha_valid[b, :n] = True
        self.alpha_count = max((len(x) for x in sel.keep), default=0)
        self.alpha_spans, self.alpha_positions = sel.spans, sel.positions
        counts = np.asarray([len(a) for a in sel.archive], np.int64)
        width = int(counts.max(initial=0))
        self.trace.append(dict(cut=cut, scores=scores, selection=sel))
        if not width:
            return
        ak = np.zeros((B, G, width, D), F32)
        av = np.zeros((B, G, width, D), F32)
        ap = np.zeros((B, width), np.int64)
        for b, arch in enumerate(sel.archive):
            n = len(arch)
            ak[b, :, :n] = keys[b][:, arch]
            av[b, :, :n] = vals[b][:, arch]
            ap[b, :n] = pos[b, arch]
        if not counts.any():
            return
        if self.unified:
            self.route_unified(ak, av, ap, counts)
        else:
            self.route_attach(ak, av, ap, counts)

    # ------------------------------------------------------------------ route
    def route_attach(self, ak, av, ap, counts):
        B, G = self.batch, self.groups
        assign, order = attach_decide(ak, ap, ap, counts, self.centroid, self.alive, self.p_hi_c, self.s_h,
                                      self.eta, self.g0, self.lam)
        self.trace[-1].update(assign=assign, order=order)
        # Group by (lane, cluster), tokens in position order (_semantic_attach_commit).
        new_jobs, jobs = [], []
        for b in range(B):
            offs = order[b, :counts[b]]
            for g in range(G):
                clusters = assign[b, g, :counts[b]].astype(np.int64)
                for c in range(self.K):
                    toks = offs[clusters == c]
                    if not len(toks):
                        continue
                    if not self.alive[b, g, c]:
                        new_jobs.append((b, g, c, int(toks[0])))
                        toks = toks[1:]
                    if len(toks):
                        jobs.append((b, g, c, [int(t) for t in toks]))
        self._commit(new_jobs, jobs, ak, av, ap)

    def _commit(self, new_jobs, jobs, ak, av, ap):
        """New clusters, then joins by (b, g, cluster), delayed when a token precedes p_hi
        (_semantic_new_clusters :2268-2298, _alpha_commit_joins :3690-3788)."""
        for b, g, c, t in new_jobs:
            self._new_cluster(b, g, c, ak[b, g, t], av[b, g, t], int(ap[b, t]))
        for b, g, c, toks in sorted(jobs, key=lambda j: j[:3]):
            tpos = ap[b, toks]
            if tpos.min() < self.p_hi_c[b, g, c]:
                self._late_join(b, g, c, ak[b, g, toks], av[b, g, toks], tpos)
            else:
                self._join(b, g, c, ak[b, g, toks], av[b, g, toks], tpos)

    def route_unified(self, ak, av, ap, counts):
        """_semantic_route_unified (log_kv_cache.py:3589-3688): per lane a radius-limited candidate
        pass over the flushed tokens, then a global pass over [live centroids, candidates] down to
        K clusters; merges of two old clusters rebuild the keep cluster's ladder (Ward merges, in
        trace order), candidates joined to an old root join that cluster, the others open new
        clusters in the free slots."""
        B, G, D, K = self.batch, self.groups, self.dim, self.K
        lanes = [(b, g) for b in range(B) for g in range(G) if counts[b]]
        if not lanes:
            return
        tile = U.route_tile(len(lanes), int(max(counts)))
        position_order = [np.argsort(ap[b, :counts[b]], kind="stable") for b in range(B)]
        routes, merge_jobs, decisions = [], [], {}
        for start in range(0, len(lanes), tile):
            part = lanes[start:start + tile]
            ccounts = [int(counts[b]) for b, _ in part]
            tokens = max(ccounts)
            mu = np.zeros((len(part), tokens, D), F32)
            for i, (b, g) in enumerate(part):
                mu[i, :ccounts[i]] = ak[b, g, :ccounts[i]].astype(F32)
            cweights = (np.arange(tokens)[None, :] < np.asarray(ccounts)[:, None]).astype(F32)
            limits = [float(np.float32(math.sqrt(self.lam * float(self.s_h[b, g])))) for b, g in part]
            candidates, ctraces = U.reduce_lanes(mu, ccounts, cweights, target=1, radius_limits=limits)
            live = [np.flatnonzero(self.alive[b, g]).astype(np.int64) for b, g in part]
            labels = U.labels_batch(ccounts, candidates, ctraces)
            weights = [np.concatenate((self.n_total[b, g, old].astype(F32),
                                       np.bincount(lab, minlength=len(roots)).astype(F32)))
                       for (b, g), old, roots, lab in zip(part, live, candidates, labels)]
            gcounts = [len(w) for w in weights]
            size = max(gcounts)
            centers = np.zeros((len(part), size, D), F32)
            padded = np.zeros((len(part), size), F32)
            for i, ((b, g), old, roots) in enumerate(zip(part, live, candidates)):
                centers[i, :len(old)] = self.centroid[b, g, old]
                centers[i, len(old):gcounts[i]] = mu[i, roots]
                padded[i, :gcounts[i]] = weights[i]
            groots, gtraces = U.reduce_lanes(centers, gcounts, padded, target=K, strict=True,
                                             passes=self.merge_passes)
            merged = U.labels_batch(gcounts, groots, gtraces)
            for (b, g), old, clab, roots, trace, lab in zip(part, live, labels, groots, gtraces, merged):
                old_trace = trace[trace[:, 1] < len(old)] if len(trace) else trace
                merge_jobs.append((b, g, [tuple(int(x) for x in pair) for pair in old[old_trace]]))
                routes.append((b, g, old, lab[len(old) + clab], roots))
                decisions[(b, g)] = dict(candidates=len(candidates[part.index((b, g))]), ctrace=ctraces[
                    part.index((b, g))], gtrace=trace, assign=lab[len(old) + clab])
        self.trace[-1].update(unified=decisions)
        for step in range(max((len(p) for _, _, p in merge_jobs), default=0)):
            for b, g, pairs in merge_jobs:
                if step < len(pairs):
                    self._ward_merge(b, g, *pairs[step])
        new_jobs, jobs = [], []
        for b, g, old, assignment, roots in routes:
            free = iter(np.flatnonzero(~self.alive[b, g]).tolist())
            order = position_order[b]
            by_cluster = assignment[order]
            perm = np.argsort(by_cluster, kind="stable")
            grouped = order[perm]
            bounds = np.searchsorted(by_cluster[perm], np.arange(len(roots) + 1))
            for cluster, root in enumerate(roots):
                offsets = grouped[bounds[cluster]:bounds[cluster + 1]]
                if not len(offsets):
                    continue
                if root < len(old):
                    target = int(old[root])
                else:
                    target = next(free)
                    new_jobs.append((b, g, target, int(offsets[0])))
                    offsets = offsets[1:]
                if len(offsets):
                    jobs.append((b, g, target, [int(t) for t in offsets]))
        self._commit(new_jobs, jobs, ak, av, ap)

    def _ward_merge(self, b, g, keep, free):
        """One Ward merge of two old clusters (_semantic_ward_merge_batch :2517-2593): the keep
        and free entries in ward_entry_index order are re-appended to the cleared keep cluster
        with orders 0..n-1; centroid the count-weighted mean."""
        ek, ef = self.ladder.entries(b, g, keep), self.ladder.entries(b, g, free)
        rows = Rows.cat(ek, ef)
        idx = U.ward_entry_index(rows.order, rows.lo, rows.w > 0, len(ek))
        rows = rows.take(idx)
        rows.order = np.arange(len(rows), dtype=np.int64)
        nk, nf = F32(self.n_total[b, g, keep]), F32(self.n_total[b, g, free])
        mu = ((((nk * self.centroid[b, g, keep]).astype(F32) + (nf * self.centroid[b, g, free]).astype(F32))
               .astype(F32)) / max(F32(nk + nf), F32(1))).astype(F32)
        ne = F32(self.n_eff[b, g, keep] + self.n_eff[b, g, free])
        total = int(self.n_total[b, g, keep] + self.n_total[b, g, free])
        hi = max(int(self.p_hi_c[b, g, keep]), int(self.p_hi_c[b, g, free]))
        for c in (keep, free):
            self.ladder.clear_lane(b, g, c)
            self.alive[b, g, c] = False
            self.n_total[b, g, c] = 0
            self.p_hi_c[b, g, c] = -1
            self.level0_phase[b, g, c] = 0
        self.centroid[b, g, keep] = mu
        self.n_eff[b, g, keep] = ne
        self.n_eff[b, g, free] = 0
        self.alive[b, g, keep] = True
        self.n_total[b, g, keep] = total
        self.p_hi_c[b, g, keep] = hi
        self.level0_phase[b, g, keep] = len(rows)
        self.ladder.append(b, g, keep, rows, self.beta)

    def _new_cluster(self, b, g, c, k, v, pos):
        self.ladder.clear_lane(b, g, c)
        self.centroid[b, g, c] = k.astype(F32)
        self.n_eff[b, g, c] = 1.0
        self.ladder.append(b, g, c, Rows.tokens(k[None], v[None], [pos], [0]), self.beta)
        self.alive[b, g, c] = True
        self.n_total[b, g, c] = 1
        self.p_hi_c[b, g, c] = pos
        self.level0_phase[b, g, c] = 1

    def _join(self, b, g, c, k, v, pos):
        """Ordinary join: tokens appended with phases, then the sequential centroid update."""
        n = len(pos)
        phase = int(self.level0_phase[b, g, c])
        self.ladder.append(b, g, c, Rows.tokens(k, v, pos, phase + np.arange(n)), self.beta)
        self.level0_phase[b, g, c] = phase + n
        self.p_hi_c[b, g, c] = int(pos[-1])
        self.n_total[b, g, c] += n
        sums = seq_sum(k.astype(F32))
        pre = F32(self.n_eff[b, g, c] * F32(1.0))
        denom = F32(pre + F32(n))
        mu = self.centroid[b, g, c]
        if pre > 0:
            self.centroid[b, g, c] = (((pre * mu).astype(F32) + sums).astype(F32) / denom).astype(F32)
        else:
            self.centroid[b, g, c] = (sums / F32(n)).astype(F32)
        self.n_eff[b, g, c] = denom

    def _late_join(self, b, g, c, k, v, pos):
        """Delayed archival: re-append every entry of the lane merged by position (_alpha_commit_joins)."""
        n = len(pos)
        old = self.ladder.entries(b, g, c)
        new = Rows.tokens(k, v, pos, np.zeros(n, np.int64))
        combined = Rows.cat(old, new)
        idx = np.argsort(combined.lo, kind="stable")
        rows = combined.take(idx)
        rows.order = np.arange(len(rows), dtype=np.int64)
        sums = seq_sum(k.astype(F32))
        pre = self.n_eff[b, g, c]
        mu = self.centroid[b, g, c]
        self.centroid[b, g, c] = (((pre * mu).astype(F32) + sums).astype(F32) / F32(pre + F32(n))).astype(F32)
        self.n_eff[b, g, c] = F32(pre + F32(n))
        total = int(self.n_total[b, g, c]) + n
        high = max(int(self.p_hi_c[b, g, c]), int(pos.max()))
        self.ladder.clear_lane(b, g, c)
        self.ladder.append(b, g, c, rows, self.beta)
        self.alive[b, g, c] = True
        self.n_total[b, g, c] = total
        self.p_hi_c[b, g, c] = high
        self.level0_phase[b, g, c] = len(rows)

    # ------------------------------------------------------------------ views
    def state(self) -> dict:
        """Arrays named like the reference buffers and host mirrors."""
        L = self.ladder
        return dict(level_k=L.k, level_v=L.v, level_w=L.w, level_p_lo=L.lo, level_p_hi=L.hi,
                    level_sum_wp=L.swp, level_order=L.order, pad_mask=L.pad, level_count=L.count,
                    centroid=self.centroid, n_eff=self.n_eff, n_total=self.n_total, p_hi_c=self.p_hi_c,
                    level0_phase=self.level0_phase, alive=self.alive,
                    recent_k=self.recent_k, recent_k_raw=self.recent_k_raw, recent_v=self.recent_v,
                    recent_pos=self.recent_pos, alpha_k_raw=self.alpha_k_raw, alpha_v=self.alpha_v,
                    alpha_pos=self.alpha_pos, alpha_valid=self.alpha_valid)
