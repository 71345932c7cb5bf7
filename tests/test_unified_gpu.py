"""Unified-route operators on the GPU against the reference's reducer and the oracle.

``UnifiedReduce`` runs the golden cases (tests/golden/unified_*.npz: the reference's
``_UnifiedReduceTorch`` to completion) and must end with the same merges in the same order,
the same survivors, stuck flags, live counts, masses, centres and distances (atol = 0);
larger random cases (with and without radius limits) are compared with the oracle the same
way, and ``pair_distances`` / ``mirror`` with the oracle's.
"""
from __future__ import annotations

import os

import numpy as np
import pytest
import torch

from oracle import unified as U

pytestmark = pytest.mark.gpu
HERE = os.path.dirname(os.path.abspath(__file__))


def run_device(dist, mu, mass, count, limits, target):
    from logkv_b200.plugin import UnifiedReduce
    t = lambda a, dt=torch.float32: torch.from_numpy(np.ascontiguousarray(a)).to("cuda", dt)  # noqa: E731
    d, m, w = t(dist), t(mu), t(mass)
    red = UnifiedReduce(d, m, w, t(count, torch.int64), None if limits is None else t(limits), target)
    for r in range(1, 2 * mass.shape[1] + 8):
        if not bool(red.step(r).any()):
            break
    traces, alive, stuck = red.finish()
    return traces, alive, stuck, red.count.cpu().numpy(), w.cpu().numpy(), m.cpu().numpy(), d.cpu().numpy()


def check(got, traces, alive, stuck, count, mass, mu, dist):
    gt, ga, gs, gc, gw, gm, gd = got
    for lane, t in enumerate(traces):
        np.testing.assert_array_equal(gt[lane], t, err_msg=f"lane {lane} traces")
    np.testing.assert_array_equal(ga, alive)
    np.testing.assert_array_equal(gs, stuck)
    np.testing.assert_array_equal(gc, count)
    np.testing.assert_array_equal(gw, mass)
    np.testing.assert_array_equal(gm, mu)
    np.testing.assert_array_equal(gd, dist)


@pytest.mark.parametrize("name", ["global", "global_wide", "candidate"])
def test_unified_reduce_matches_reference(name):
    f = np.load(os.path.join(HERE, "golden", f"unified_{name}.npz"))
    limits = f["in_limits"] if "in_limits" in f.files else None
    got = run_device(f["in_dist"], f["in_mu"], f["in_mass"], f["in_count"], limits, int(f["target"]))
    traces = [f[f"trace{lane}"] for lane in range(f["in_mass"].shape[0])]
    check(got, traces, f["alive"], f["stuck"], f["count"], f["mass"], f["mu"], f["dist"])


def random_case(seed, L, M, D, limited):
    rng = np.random.default_rng(seed)
    centres = rng.standard_normal((L, 9, D)).astype(np.float32) * 2
    z = rng.integers(0, 9, (L, M))
    mu = (centres[np.arange(L)[:, None], z] + 0.4 * rng.standard_normal((L, M, D))).astype(np.float32)
    count = rng.integers(M // 2, M + 1, L)
    count[0] = M
    live = np.arange(M)[None, :] < count[:, None]
    mass = np.where(live, 1.0 if limited else rng.integers(1, 9, (L, M)), 0).astype(np.float32)
    mu = np.where(live[..., None], mu, 0).astype(np.float32)
    c = (mu - mu[:, :1]).astype(np.float32)
    norm = np.zeros((L, M), np.float32)
    for d in range(D):
        norm = (norm + (c[..., d] * c[..., d]).astype(np.float32)).astype(np.float32)
    gram = np.einsum("lid,ljd->lij", c.astype(np.float64), c.astype(np.float64)).astype(np.float32)
    dist = U.pair_distances(gram, norm)
    limits = (rng.random(L) * 1.5 + 1.0).astype(np.float32) if limited else None
    return dist, mu, mass, count, limits


@pytest.mark.parametrize("limited", [False, True])
@pytest.mark.parametrize("L,M,D", [(4, 300, 64), (1, 1500, 32)])
def test_unified_reduce_matches_oracle_random(limited, L, M, D):
    dist, mu, mass, count, limits = random_case(11 + limited + M, L=L, M=M, D=D, limited=limited)
    target = 1 if limited else 12
    red = U.UnifiedReduce(dist, mu, mass, count, limits, target)
    for _ in range(2 * M + 8):
        if not red.step().any():
            break
    traces, alive, stuck = red.finish()
    got = run_device(dist, mu, mass, count, limits, target)
    check(got, traces, alive, stuck, red.count, red.mass, red.mu, red.dist)


def test_pair_distances_and_mirror_match_oracle():
    from logkv_b200.plugin import mirror, pair_distances
    rng = np.random.default_rng(5)
    gram = rng.standard_normal((3, 77, 77)).astype(np.float32)
    norm = (rng.random((3, 77)) * 4).astype(np.float32)
    got = pair_distances(torch.from_numpy(gram.copy()).cuda(), torch.from_numpy(norm).cuda()).cpu().numpy()
    np.testing.assert_array_equal(got, U.pair_distances(gram, norm))
    got = mirror(torch.from_numpy(gram.copy()).cuda()).cpu().numpy()
    np.testing.assert_array_equal(got, U.mirror(gram))
