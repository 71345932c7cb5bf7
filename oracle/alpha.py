"""Alpha exact-span pool selection (TEST INFRASTRUCTURE ONLY).

Restates litgpt/alpha_log_kv.py: the span cut (``_new_runs`` :16-53 and
``cut_spans`` :84-122), the span scores including Beta's novelty (``score_spans``
:125-174) and the bounded whole-span greedy (``choose_spans`` :177-226).

Candidates of one batch row index tokens of [old pool padded to ``old_width`` |
current flush], shared by every KV group of the row.
"""
from __future__ import annotations

from dataclasses import dataclass, field

import numpy as np

from .numerics import F32, ddot, dsum


@dataclass
class Candidate:
    ranges: list          # [(start, stop)] token ranges into [pool | flush]
    old: bool             # a closed span already in the pool
    closed: bool          # False only for the mandatory unfinished tail

    @property
    def length(self) -> int:
        return sum(b - a for a, b in self.ranges)

    def tokens(self) -> list:
        out = []
        for a, b in self.ranges:
            out.extend(range(a, b))
        return out


@dataclass
class RowCut:
    candidates: list
    positions: np.ndarray      # [old_width + T] positions of [pool | flush]


@dataclass
class Selection:
    keep: list = field(default_factory=list)        # per row: kept token indices
    archive: list = field(default_factory=list)     # per row: archived token indices
    spans: list = field(default_factory=list)       # per row: [(length, closed)]
    positions: list = field(default_factory=list)   # per row: kept positions


def new_runs(pos, ends, pending: int, pending_pos: int, max_span: int):
    """Runs of the new tokens of one row (alpha_log_kv._new_runs, :16-53).

    A run closes after a span boundary or when it reaches ``max_span`` tokens
    (counting the unfinished old span it continues), and before a position jump.
    Returns (pending_closed, starts, stops, closed).
    """
    pos = np.asarray(pos, dtype=np.int64)
    end = np.asarray(ends, dtype=bool)
    n = len(pos)
    if n == 0:
        return False, [], [], []
    pending_closed = bool(pending) and int(pos[0]) != pending_pos + 1
    prefix = 0 if pending_closed else pending
    starts, stops, closed = [], [], []
    run_start = 0
    seg_first = 0
    first_segment = True
    for i in range(n):
        if i > 0 and (pos[i] != pos[i - 1] + 1 or end[i - 1]):
            seg_first = i
            first_segment = False
        filled = i - seg_first + (prefix if first_segment else 0) + 1
        cap = filled % max_span == 0
        if prefix >= max_span and first_segment:
            cap = False
        close = bool(end[i]) or cap
        jump_next = i + 1 < n and pos[i + 1] != pos[i] + 1
        if close or jump_next or i == n - 1:
            starts.append(run_start)
            stops.append(i + 1)
            closed.append(close or jump_next)
            run_start = i + 1
    return pending_closed, starts, stops, closed


def cut_spans(old_spans, old_positions, new_positions, ends, old_width: int, max_span: int):
    """Whole candidate spans per row, or None when no row has any (cut_spans, :84-122)."""
    rows = []
    any_tokens = False
    for spans, old_pos, new_pos, boundaries in zip(old_spans, old_positions, new_positions, ends):
        cands, offset, pending = [], 0, None
        for length, closed in spans:
            if closed:
                cands.append(Candidate([(offset, offset + length)], True, True))
            else:
                pending = (offset, offset + length)
            offset += length
        all_pos = np.zeros(old_width + len(new_pos), dtype=np.int64)
        all_pos[:len(old_pos)] = old_pos
        all_pos[old_width:] = new_pos
        pending_len = 0 if pending is None else pending[1] - pending[0]
        pclosed, starts, stops, closed = new_runs(
            new_pos, boundaries, pending_len, int(all_pos[pending[1] - 1]) if pending_len else 0, max_span)
        if pclosed:
            cands.append(Candidate([pending], False, True))
        for i, (a, b, done) in enumerate(zip(starts, stops, closed)):
            ranges = [(a + old_width, b + old_width)]
            if i == 0 and pending_len and not pclosed:
                ranges.insert(0, pending)
            cands.append(Candidate(ranges, False, bool(done)))
        if pending_len and not pclosed and not starts:
            cands.append(Candidate([pending], False, False))
        any_tokens |= any(c.length for c in cands)
        rows.append(RowCut(cands, all_pos))
    return rows if any_tokens else None


def _span_parts(x: np.ndarray, tokens: list):
    """Per-group (mean vector, energy) of one span; x is [G, N, D] float32."""
    xs = x[:, tokens, :].astype(F32)                         # [G, n, D]
    n = F32(len(tokens))
    acc = np.zeros((x.shape[0], x.shape[2]), F32)
    for t in range(xs.shape[1]):
        acc = (acc + xs[:, t]).astype(F32)
    mean = (acc / n).astype(F32)                              # [G, D]
    per_tok = (dsum((xs * xs).astype(F32)) / F32(x.shape[2])).astype(F32)   # [G, n]
    e = np.zeros(x.shape[0], F32)
    for t in range(per_tok.shape[1]):
        e = (e + per_tok[:, t]).astype(F32)
    energy = (e / n).astype(F32)                              # [G]
    return mean, energy


def score_spans(keys, values, cut, *, beta_novelty=False, centroids=None, centroid_valid=None):
    """Scores per row and candidate (score_spans, :125-174), as Python floats.

    keys/values: [B, G, N, D] float32 of [pool | flush].  Alpha: mean over
    groups of R_K + R_V with R = max(E - mean(mu^2), 0) / max(E, 1e-12).
    Beta: per group (R_K+R_V)/2 + N/(1+N) with N the nearest live centre's
    mean-square distance over E_K, then the mean of the top-min(2, G) groups.
    """
    out = []
    G, D = keys.shape[1], keys.shape[3]
    for b, rowcut in enumerate(cut):
        row_scores = []
        for cand in rowcut.candidates:
            toks = cand.tokens()
            if not toks:
                row_scores.append(0.0)
                continue
            parts = []
            kmean = kenergy = kms = None
            for comp, src in enumerate((keys, values)):
                mean, energy = _span_parts(src[b], toks)
                ms = (dsum((mean * mean).astype(F32)) / F32(D)).astype(F32)
                resid = np.maximum((energy - ms).astype(F32), F32(0))
                part = (resid / np.maximum(energy, F32(1e-12))).astype(F32)
                if comp == 0:
                    kmean, kenergy, kms = mean, energy, ms
                parts.append(part)
            if not beta_novelty:
                s = ((dsum(parts[0]) / F32(G)).astype(F32) + (dsum(parts[1]) / F32(G)).astype(F32)).astype(F32)
                row_scores.append(float(F32(s)))
                continue
            score = (parts[0] + parts[1]).astype(F32)                        # [G]
            mu = centroids[b].astype(F32)                                    # [G, K, D]
            dots = (ddot(kmean[:, None, :], mu) / F32(D)).astype(F32)
            mm = (dsum((mu * mu).astype(F32)) / F32(D)).astype(F32)  # [G, K]
            dist = np.maximum(((kms[:, None] + mm).astype(F32) - (F32(2) * dots)).astype(F32), F32(0))
            valid = centroid_valid[b].astype(bool)
            nearest = np.where(valid, dist, np.inf).min(axis=-1).astype(F32)
            nearest = np.where(valid.any(-1), nearest, F32(0)).astype(F32)
            novelty = (nearest / np.maximum(kenergy, F32(1e-12))).astype(F32)
            score = ((score * F32(0.5)).astype(F32) + (novelty / (F32(1) + novelty)).astype(F32)).astype(F32)
            top = np.sort(score)[::-1][:min(2, G)]
            row_scores.append(float(F32(dsum(top) / F32(len(top)))))
        out.append(row_scores)
    return out


def choose_spans(cut, scores, budget: int) -> Selection:
    """Bounded whole-span greedy per row (choose_spans, :177-226), in float64 like the host code."""
    sel = Selection()
    for rowcut, row_scores in zip(cut, scores):
        cands = rowcut.candidates
        size = [c.length for c in cands]
        density = [row_scores[i] * (1.1 if c.old else 1.0) for i, c in enumerate(cands)]
        mandatory = {i for i, c in enumerate(cands) if not c.closed}
        room = budget - sum(size[i] for i in mandatory)
        chosen = mandatory | {i for i, c in enumerate(cands) if c.old}
        room -= sum(size[i] for i in chosen - mandatory)

        def victims():
            return sorted(chosen - mandatory, key=lambda i: (density[i], -i))

        for i in victims():
            if room >= 0:
                break
            chosen.remove(i)
            room += size[i]
        ranked = sorted((i for i in range(len(cands)) if i not in chosen), key=lambda i: (-density[i], i))
        order = None
        for i in ranked:
            length = size[i]
            available, loss, remove = room, 0.0, []
            if available < length:
                if order is None:
                    order = victims()
                for j in order:
                    remove.append(j)
                    available += size[j]
                    loss += density[j] * size[j]
                    if available >= length:
                        break
            if available >= length and (not remove or density[i] * length > loss):
                chosen.difference_update(remove)
                chosen.add(i)
                room = available - length
                order = None
        selected = sorted(chosen)
        keep, archive = [], []
        for i, c in enumerate(cands):
            (keep if i in chosen else archive).extend(c.tokens())
        sel.keep.append(keep)
        sel.archive.append(archive)
        sel.spans.append([(size[i], cands[i].closed) for i in selected])
        sel.positions.append([int(rowcut.positions[t]) for t in keep])
    return sel
