"""Golden cases for the unified (Ward / radius) reducer, from the UNMODIFIED reference on CPU.

Test infrastructure only (same import shim as make_golden.py).  Seeded cases: clustered centres
with integer masses reduced to a target without radius limits (the global pass), and unit-mass
tokens reduced toward one cluster under per-lane radius limits (the candidate pass).  Inputs are
squared distances from the reference's own pair matrix (``_semantic_unified_pair_matrix``,
log_kv_cache.py:3185-3221), centres, masses, counts, limits; outputs are the reference
``_UnifiedReduceTorch`` (:448-638) results after running its rounds to the end: merge traces,
alive flags, stuck flags, final masses, centres and distances.

Usage:  python tests/golden/make_unified.py --reference <checkout> [--out tests/golden]
"""
from __future__ import annotations

import argparse
import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, HERE)
from make_golden import install_shim  # noqa: E402

CASES = [
    dict(name="global", lanes=3, size=48, counts=(48, 40, 31), dim=16, target=6, limits=None, seed=1),
    dict(name="global_wide", lanes=2, size=96, counts=(96, 77), dim=32, target=12, limits=None, seed=2),
    dict(name="candidate", lanes=3, size=64, counts=(64, 50, 40), dim=16, target=1, limits=(1.6, 2.2, 1.2), seed=3),
]


def make_case(c):
    g = torch.Generator().manual_seed(c["seed"])
    L, M, D = c["lanes"], c["size"], c["dim"]
    centres = torch.randn(L, 6, D, generator=g) * 2.0
    z = torch.randint(0, 6, (L, M), generator=g)
    mu = (centres[torch.arange(L)[:, None], z] + 0.35 * torch.randn(L, M, D, generator=g)).float()
    counts = torch.tensor(c["counts"], dtype=torch.int64)
    live = torch.arange(M)[None, :] < counts[:, None]
    if c["limits"] is None:
        mass = torch.randint(1, 6, (L, M), generator=g).float()
    else:
        mass = torch.ones(L, M)
    mass = torch.where(live, mass, torch.zeros_like(mass))
    mu = torch.where(live[..., None], mu, torch.zeros_like(mu))
    return mu, mass, counts


def run(case):
    from litgpt.log_kv_cache import LogStructuredKVCache, _UnifiedReduceTorch
    mu, mass, counts = make_case(case)
    dist = LogStructuredKVCache._semantic_unified_pair_matrix(mu.clone())
    limits = None if case["limits"] is None else torch.tensor(case["limits"], dtype=torch.float32)
    out = {"in_dist": dist.numpy().copy(), "in_mu": mu.numpy().copy(), "in_mass": mass.numpy().copy(),
           "in_count": counts.numpy().copy(), "target": np.int64(case["target"])}
    if limits is not None:
        out["in_limits"] = limits.numpy().copy()
    red = _UnifiedReduceTorch(dist.clone(), mu.clone(), mass.clone(), counts.clone(), limits, case["target"], 1)
    rounds = 0
    for r in range(1, 2 * case["size"] + 8):
        rounds = r
        if not bool(red.step(r).any()):
            break
    traces, alive, stuck = red.finish()
    for lane, t in enumerate(traces):
        out[f"trace{lane}"] = np.asarray(t, np.int64).reshape(-1, 2)
    out.update(alive=alive, stuck=stuck, mass=red.mass.numpy(), mu=red.mu.numpy(), dist=red.dist.numpy(),
               count=red.count.numpy(), rounds=np.int64(rounds))
    return out


def main():
    parser = argparse.ArgumentParser()
    parser.add_argument("--reference", default=os.environ.get("LOGKV_REFERENCE"))
    parser.add_argument("--out", default=HERE)
    args = parser.parse_args()
    if not args.reference:
        raise SystemExit("pass --reference <reference checkout> or set LOGKV_REFERENCE")
    install_shim(args.reference)
    torch.set_num_threads(1)
    for case in CASES:
        out = run(case)
        path = os.path.join(args.out, f"unified_{case['name']}.npz")
        np.savez_compressed(path, **out)
        print("wrote", path, os.path.getsize(path), "rounds", int(out["rounds"]), "count", out["count"].tolist())


if __name__ == "__main__":
    main()
