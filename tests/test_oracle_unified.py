"""The unified-route oracle against the reference's own reducer (tests/golden/unified_*.npz).

The fixtures hold inputs and the end state of the reference's ``_UnifiedReduceTorch`` run to
completion; the oracle must make the same merges in the same order, leave the same clusters
alive and end with the same masses, centres and distances (atol = 0).  The one sum the
reference leaves to torch's CPU order (the exact squared distance checked against a radius
limit) runs left to right in the oracle; the candidate case checks that no decision depends on it.
"""
from __future__ import annotations

import os

import numpy as np
import pytest

from oracle import unified as U

HERE = os.path.dirname(os.path.abspath(__file__))
CASES = ["global", "global_wide", "candidate"]


def load(name):
    return np.load(os.path.join(HERE, "golden", f"unified_{name}.npz"))


def run_oracle(f):
    limits = f["in_limits"] if "in_limits" in f.files else None
    red = U.UnifiedReduce(f["in_dist"], f["in_mu"], f["in_mass"], f["in_count"], limits, int(f["target"]))
    for _ in range(2 * f["in_mass"].shape[1] + 8):
        if not red.step().any():
            break
    return red


@pytest.mark.parametrize("name", CASES)
def test_oracle_matches_reference_reducer(name):
    f = load(name)
    red = run_oracle(f)
    traces, alive, stuck = red.finish()
    for lane, t in enumerate(traces):
        np.testing.assert_array_equal(t, f[f"trace{lane}"], err_msg=f"lane {lane} traces")
    np.testing.assert_array_equal(alive, f["alive"])
    np.testing.assert_array_equal(stuck, f["stuck"])
    np.testing.assert_array_equal(red.count, f["count"])
    np.testing.assert_array_equal(red.mass, f["mass"])
    np.testing.assert_array_equal(red.mu, f["mu"])
    np.testing.assert_array_equal(red.dist, f["dist"])


def test_pair_distances_and_mirror():
    rng = np.random.default_rng(0)
    L, M = 2, 40
    gram = rng.standard_normal((L, M, M)).astype(np.float32)
    norm = rng.random((L, M)).astype(np.float32) * 4
    d = U.pair_distances(gram, norm)
    assert np.array_equal(d, np.transpose(d, (0, 2, 1)))
    i, j = 3, 17
    want = max(np.float32(np.float32(norm[1, i] + norm[1, j]) - np.float32(2) * gram[1, i, j]), np.float32(0))
    assert d[1, i, j] == want
    m = U.mirror(gram)
    assert np.array_equal(m[0][np.triu_indices(M)], gram[0][np.triu_indices(M)])
    assert np.array_equal(m, np.transpose(m, (0, 2, 1)))


def test_fma32_is_correctly_rounded():
    """The oracle's float32 fused multiply-add (the Gram products' form) equals a * b + c rounded
    once to the nearest float32 (ties to even), against exact rational arithmetic: random
    operands, cancellations, and sums lying exactly on a float32 midpoint in float64."""
    from fractions import Fraction

    def exact_round(a, b, c):
        v = Fraction(float(a)) * Fraction(float(b)) + Fraction(float(c))
        f = np.float32(float(v))
        cands = [np.nextafter(f, np.float32(-np.inf)), f, np.nextafter(f, np.float32(np.inf))]
        return min(cands, key=lambda t: (abs(Fraction(float(t)) - v), int(np.array(t).view(np.uint32)) & 1))

    rng = np.random.default_rng(5)
    a = rng.standard_normal(3000).astype(np.float32)
    b = rng.standard_normal(3000).astype(np.float32)
    c = rng.standard_normal(3000).astype(np.float32)
    cancel = (-(a.astype(np.float64) * b.astype(np.float64))).astype(np.float32)
    # Double-rounding cases: a * b = 2^-24 (1 - 2^-46) exactly, so c + a * b rounds in float64
    # onto the float32 midpoint c + 2^-24 although the exact sum lies just below it; with c odd
    # (1 + 2^-23) ties-to-even from that midpoint would round up, the correct result is c.
    a_mid = np.full(4, np.float32(1.0 + 2.0 ** -23), np.float32)
    b_mid = np.asarray([2.0 ** -24 * (1 - 2.0 ** -23), -2.0 ** -24 * (1 - 2.0 ** -23)] * 2, np.float32)
    c_mid = np.asarray([1.0, -1.0, 1.0 + 2.0 ** -23, -(1.0 + 2.0 ** -23)], np.float32)
    for x, y, z in ((a, b, c), (a, b, cancel), (a_mid, b_mid, c_mid)):
        got = U.fma32(x, y, z)
        want = np.asarray([exact_round(p, q, r) for p, q, r in zip(x, y, z)], np.float32)
        np.testing.assert_array_equal(got.view(np.uint32), want.view(np.uint32))
    # The last case is one that a plain float64 sum rounded to float32 gets wrong.
    naive = (a_mid.astype(np.float64) * b_mid.astype(np.float64) + c_mid.astype(np.float64)).astype(np.float32)
    assert not np.array_equal(naive.view(np.uint32), U.fma32(a_mid, b_mid, c_mid).view(np.uint32))
