"""Batched flushes (one span-part exchange for many caches) equal plain add_recent, bit for bit.

``logkv_b200.sharding.BatchedFlush`` splits every cache's flush at its span-part exchange
(``add_recent_deferred`` / ``commit_deferred``) so that a model's layers exchange their parts in
one collective per chunk.  On one GPU (no exchange) three caches fed three seeded golden streams
through the batch, on per-layer streams, must end every chunk with the same buffers and host
mirrors as three caches fed the same chunks through ``add_recent``.
"""
from __future__ import annotations

import pytest
import torch

from fixtures import config, make_stream
from test_flush_gpu import FIELDS, make_cache, torch_dtype

pytestmark = pytest.mark.gpu


def chunk_kwargs(cfg, chunk):
    dt = torch_dtype(cfg)
    return dict(k=torch.from_numpy(chunk["k"]).to("cuda", dt), v=torch.from_numpy(chunk["v"]).to("cuda", dt),
                k_raw=torch.from_numpy(chunk["k_raw"]).to("cuda", dt),
                input_pos=torch.from_numpy(chunk["pos"]).cuda() if chunk.get("pos") is not None else None,
                span_ends=chunk["span_ends"].tolist())


@pytest.mark.parametrize("name", ["bf16_beta", "fp32_beta_sh"])
def test_batched_flush_equals_add_recent(name, cascade_path):
    from logkv_b200.sharding import BatchedFlush
    cfg = config(name)
    streams = [make_stream(dict(cfg, seed=cfg["seed"] + 10 * i)) for i in range(3)]
    plain = [make_cache(cfg, st) for st in streams]
    batched = [make_cache(cfg, st) for st in streams]
    batch = BatchedFlush(batched)
    side = [torch.cuda.Stream() for _ in range(3)]
    flushed = 0
    for step in range(len(streams[0]["chunks"])):
        kws = [chunk_kwargs(cfg, st["chunks"][step]) for st in streams]
        for cache, kw in zip(plain, kws):
            cache.add_recent(**kw)
        flushed += batch.add_recent(kws, side)
        batch.wait_all()
        torch.cuda.synchronize()
        for i, (a, b) in enumerate(zip(plain, batched)):
            assert b.read_status() == 0
            for field in FIELDS:
                assert torch.equal(getattr(a, field), getattr(b, field)), (step, i, field)
            assert a._alpha_spans == b._alpha_spans and a.alpha_count == b.alpha_count, (step, i)
            assert (a.recent_count, a.token_count) == (b.recent_count, b.token_count)
    assert flushed >= 10
