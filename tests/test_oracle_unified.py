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
