"""logkv_flush_chunk (one flush with the chunk written once, after the shift) against the
append-then-flush path it replaces, bit for bit.

Two caches take the same chunks of varying sizes; one lets ``add_recent`` use
logkv_flush_chunk whenever the chunk triggers one flush of rows already in the window
(window fill before the chunk in [take, 2 take]), the other always appends
(logkv_window_append) and then flushes (logkv_flush).  Chunk sizes below, equal to and above
the flush size make the kept old rows, the chunk rows and the zeroed leftovers land in every
arrangement.  After every chunk every buffer, the window fill and the Alpha span table must be
equal, and the fused path must have run on most flushes.
"""
from __future__ import annotations

import pytest
import torch

from fixtures import config, make_stream
from test_flush_gpu import FIELDS, make_cache, torch_dtype

pytestmark = pytest.mark.gpu

SIZES = [32, 32, 20, 12, 32, 7, 25, 32, 32, 16, 30, 2, 31, 1, 32, 17, 15, 32]


@pytest.mark.parametrize("name", ["bf16_beta", "fp32_beta_g2k", "fp32_beta_sh"])
def test_flush_chunk_equals_append_then_flush(name):
    cfg = dict(config(name), steps=len(SIZES), max_seq=1024)
    stream = make_stream(cfg)
    fused, plain = make_cache(cfg, stream), make_cache(cfg, stream)
    plain._chunk_flush_take = lambda n: None     # always append, then flush
    runs = {"fused": 0}
    inner = fused._flush_chunk

    def counted(chunk, take):
        runs["fused"] += 1
        inner(chunk, take)

    fused._flush_chunk = counted
    dt = torch_dtype(cfg)
    flushes = 0
    for step, n in enumerate(SIZES):
        n = min(n, cfg["recent"])
        chunk = stream["chunks"][step]
        k, kr, v = (torch.from_numpy(chunk[f][:, :, :n].copy()).to("cuda", dt) for f in ("k", "k_raw", "v"))
        ends = chunk["span_ends"][:, :n].tolist()
        before = plain._flush_cursor
        for cache in (fused, plain):
            cache.add_recent(k, v, k_raw=kr, span_ends=ends)
        flushes += plain._flush_cursor - before
        torch.cuda.synchronize()
        assert fused.read_status() == 0 and plain.read_status() == 0
        for field in FIELDS:
            assert torch.equal(getattr(fused, field), getattr(plain, field)), (step, field)
        assert torch.equal(fused._recent_ends, plain._recent_ends), step
        assert fused.recent_count == plain.recent_count and fused.token_count == plain.token_count
        assert fused._alpha_spans == plain._alpha_spans and fused.alpha_count == plain.alpha_count, step
    assert flushes >= 8
    assert runs["fused"] >= flushes // 2, (runs, flushes)
