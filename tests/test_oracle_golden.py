"""Pin the CPU oracle against the reference itself (golden streams) and its known-answer tests.

CPU only.  Every fixture was produced by the unmodified reference cache
(tests/golden/make_golden.py); the oracle replays the same seeded stream and
must reproduce every buffer and host mirror after every ``add_recent``:
integer/layout fields and ladder K/V bit for bit, decisions identical.
"""
from __future__ import annotations

import numpy as np
import pytest

from fixtures import CONFIGS, as_values, config, load, make_stream
from oracle.alpha import choose_spans, cut_spans, new_runs, score_spans
from oracle.cache import OracleCache
from oracle.ladder import Rows, beta_layout, beta_merge

EXACT = ["level_count", "alive", "p_hi_c", "n_total", "level0_phase", "level_p_lo", "level_p_hi",
         "level_sum_wp", "level_order", "pad_mask", "level_w", "alpha_pos", "alpha_valid", "recent_pos",
         "level_k", "level_v", "alpha_k_raw", "alpha_v", "recent_k", "recent_k_raw", "recent_v",
         "centroid", "n_eff"]


def oracle_for(cfg) -> OracleCache:
    return OracleCache(batch=cfg["batch"], groups=cfg["groups"], max_seq=cfg["max_seq"], dim=cfg["dim"],
                       B=cfg["slots"], recent=cfg["recent"], clusters=cfg["clusters"],
                       granularity=cfg["granularity"], exact=cfg["exact"], span_cap=cfg["span_cap"],
                       beta=cfg["beta"], dtype=cfg["dtype"], s_h=cfg.get("s_h"))


def compare_state(oc: OracleCache, ref: dict, step: int) -> None:
    st = oc.state()
    for name in EXACT:
        want = as_values(ref[name], name)
        got = np.asarray(st[name])
        if want.dtype == bool:
            got = got.astype(bool)
        np.testing.assert_array_equal(got.astype(want.dtype), want, err_msg=f"step {step} field {name}")
    assert ref["scalars"].tolist()[:3] == [oc.alpha_count, oc.recent_count, oc.token_count], step
    for b in range(oc.batch):
        n = int(ref["alpha_nspans"][b])
        spans = [(int(a), bool(c)) for a, c in ref["alpha_spans"][b, :n]]
        assert spans == [(int(a), bool(c)) for a, c in oc.alpha_spans[b]], (step, b)
        width = len(oc.alpha_positions[b])
        assert ref["alpha_positions"][b, :width].tolist() == oc.alpha_positions[b], (step, b)


@pytest.mark.parametrize("name", [c["name"] for c in CONFIGS])
def test_oracle_replays_reference_stream(name):
    cfg = config(name)
    stream = make_stream(cfg)
    ref_steps = load(name)
    oc = oracle_for(cfg)
    assert (oc.B_prime, oc.L) == tuple(ref_steps[0]["scalars"][3:5])
    for step, (chunk, ref) in enumerate(zip(stream["chunks"], ref_steps)):
        oc.add_recent(chunk["k"], chunk["v"], chunk["k_raw"], chunk["positions"], chunk["span_ends"])
        compare_state(oc, ref, step)


# ---------------------------------------------------------------- known-answer vectors of the reference's tests

def entry_rows(values, weights):
    v = np.repeat(np.asarray(values, np.float32)[:, None], 8, axis=1)
    w = np.asarray(weights, np.float32)
    pos = np.arange(len(values), dtype=np.int64)
    return Rows(np.ones_like(v), v, w, pos.copy(), pos.copy(), pos * w.astype(np.int64), pos.copy(),
                np.zeros(len(values), bool))


def test_beta_layout_and_merge_known_answer():
    # tests/test_beta_log_kv.py:45-63 of the reference.
    assert beta_layout([0, 6, 0, 2]).tolist() == [[0, 4, 0], [4, 2, 2], [6, 2, 3]]
    assert beta_layout([]).shape == (0, 3)
    block = entry_rows([10, 0, 0, 0, 7, 9, 20, 30], [1, 2, 3, 4, 1, 1, 2, 3])
    lane1, cuts1 = beta_merge(block.take(slice(0, 6)))
    lane2, cuts2 = beta_merge(block.take(slice(6, 8)))
    assert cuts1.tolist() + cuts2.tolist() == [1, 1, 1]
    w = np.concatenate([lane1.w, lane2.w])
    v0 = np.concatenate([lane1.v[:, 0], lane2.v[:, 0]])
    np.testing.assert_allclose(w, [1, 9, 2, 5])
    np.testing.assert_allclose(v0, [10, 0, 8, 26])
    assert lane1.swp.sum() + lane2.swp.sum() == block.swp.sum()
    replay, _ = beta_merge(block.take(slice(0, 6)), cuts1)
    for a, b in zip(replay.fields(), lane1.fields()):
        np.testing.assert_array_equal(a, b)


def test_beta_cut_never_worse_than_fixed_pairs():
    # tests/test_beta_log_kv.py:66-85: chosen cut's loss <= the 2|2 loss.
    from oracle.ladder import beta_cost_cut
    rng = np.random.default_rng(83)
    block = entry_rows([0] * 40, rng.integers(1, 10, 40).tolist())
    block.k = rng.standard_normal((40, 7)).astype(np.float32)
    block.v = rng.standard_normal((40, 11)).astype(np.float32)
    for start in range(0, 40, 4):
        cut, costs = beta_cost_cut(block.take(slice(start, start + 4)), 4)
        assert costs[(2, 1, 3).index(cut)] <= costs[0] + 1e-5


def test_span_runs_match_token_loop():
    # tests/test_alpha_log_kv.py:44-78: the whole-array runs equal a per-token loop.
    def loop(new_pos, ends, pending, pending_pos, max_span):
        current, out, pclosed, last = list(range(-pending, 0)), [], False, pending_pos
        for j, (pos, end) in enumerate(zip(new_pos, ends)):
            if current and pos != last + 1:
                if current[0] < 0 and current[-1] < 0:
                    pclosed = True
                else:
                    out.append((max(current[0], 0), current[-1] + 1, True))
                current = []
            current.append(j)
            last = pos
            if end or len(current) == max_span:
                out.append((max(current[0], 0), current[-1] + 1, True))
                current = []
        if current and current[-1] >= 0:
            out.append((max(current[0], 0), current[-1] + 1, False))
        return pclosed, out

    rng = np.random.default_rng(11)
    for _ in range(400):
        count, max_span = int(rng.integers(0, 30)), int(rng.integers(1, 6))
        pending = int(rng.integers(0, max_span + 2))
        steps = 1 + (rng.random(count) < .1) * rng.integers(1, 4, count)
        new_pos = (100 + np.cumsum(steps)).tolist()
        ends = (rng.random(count) < .2).tolist()
        pending_pos = new_pos[0] - int(rng.integers(1, 3)) if count else 0
        pc, starts, stops, closed = new_runs(new_pos, ends, pending, pending_pos, max_span)
        assert (pc, list(zip(starts, stops, closed))) == loop(new_pos, ends, pending, pending_pos, max_span)


def _select(k, v, old_spans, old_pos, new_pos, ends, width, budget, cap, **kw):
    cut = cut_spans(old_spans, old_pos, new_pos, ends, width, cap)
    scores = score_spans(k, v, cut, **kw)
    return choose_spans(cut, scores, budget)


def test_spans_whole_and_pending_crosses_flush_and_cap():
    # tests/test_alpha_log_kv.py:81-93.
    k = np.random.default_rng(0).standard_normal((1, 2, 7, 8)).astype(np.float32)
    r = _select(k, k, [[(2, False)]], [[0, 1]], [[2, 3, 4, 5, 6]], [[False, True, False, False, False]], 2, 7, 4)
    assert r.keep == [list(range(7))]
    assert r.spans == [[(4, True), (3, False)]]
    assert r.archive == [[]]
    k[:, :, :4] = 1.
    r = _select(k, k, [[(4, True)]], [[0, 1, 2, 3]], [[4, 5, 6]], [[False, False, True]], 4, 4, 4)
    assert r.keep == [[4, 5, 6]]
    assert r.archive == [[0, 1, 2, 3]]


def test_beta_novelty_known_answers():
    # tests/test_beta_log_kv.py:21-42.
    k = np.broadcast_to(np.array([1., 3.], np.float32).reshape(1, 1, 2, 1), (1, 4, 2, 2)).copy()
    centers = np.ones((1, 4, 2, 2), np.float32)
    valid = np.array([[[True, False]] * 4])
    args = (k, k, [[]], [[]], [[0, 1]], [[True, True]], 0, 1, 1)
    assert _select(*args).keep == [[0]]
    r = _select(*args, beta_novelty=True, centroids=centers, centroid_valid=valid)
    assert r.keep == [[1]] and r.archive == [[0]]
    assert _select(*args, beta_novelty=True, centroids=centers, centroid_valid=valid & False).keep == [[0]]
    k = np.ones((1, 4, 2, 1), np.float32)
    k[:, :2, 0] = 3.
    k[:, :, 1] = 2.
    r = _select(k, k, [[]], [[]], [[0, 1]], [[True, True]], 0, 1, 1, beta_novelty=True,
                centroids=np.ones((1, 4, 1, 1), np.float32), centroid_valid=np.ones((1, 4, 1), bool))
    assert r.keep == [[0]]


def test_delayed_archive_known_answer():
    # tests/test_alpha_log_kv.py:198-208: a late join keeps weighted positions (sum_wp = 47).
    oc = OracleCache(batch=2, groups=2, max_seq=128, dim=8, B=8, recent=8, clusters=4, granularity=8,
                     exact=8, span_cap=4, beta=False)
    k = np.random.default_rng(1).standard_normal((2, 2, 8, 8)).astype(np.float32)
    oc._new_cluster(0, 0, 0, k[0, 0, 0], k[0, 0, 0], 40)
    oc._late_join(0, 0, 0, k[0, 0, :2], k[0, 0, :2], np.array([3, 4]))
    assert oc.p_hi_c[0, 0, 0] == 40
    assert oc.ladder.w[0, 0, 0].sum() == 3
    assert oc.ladder.swp[0, 0, 0].sum() == 47
    assert oc.n_total[0, 0, 0] == 3
