"""CPU oracle for the SemanticLogKV flush-and-attend path (TEST INFRASTRUCTURE ONLY).

This package restates, in numpy, the reference's CPU Torch path for the in-scope
configuration (attach route, Alpha exact-span pool, optional Beta, mid anchors,
first-order entries).  It exists to check the CUDA product, never to serve it:
only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline leg
may import it.

Parity pin: the oracle is checked field-by-field against fixtures produced by
running the unmodified reference (``tests/golden/make_golden.py``) and against
the known-answer vectors of the reference's own tests
(``tests/test_oracle_golden.py``).

Module map (each function cites the reference lines it follows):
  numerics.py  - float32 / bfloat16 rounding helpers
  ladder.py    - per-lane ladder append, pairwise and Beta 4->2 merges, top fold
  alpha.py     - span cut, span scores (Alpha and Beta novelty), bounded greedy choice
  attach.py    - frozen-centroid attach decisions with farthest-point seeding
  cache.py     - the cache state and the whole flush (add_recent -> route -> commit)
  attention.py - mid-anchor attention plan and slot attention (math path)
"""
