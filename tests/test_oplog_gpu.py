"""Route op-log against the reference's own (tests/golden/oplog_*.npz, from make_oplog.py).

The reference cache, driven through the golden streams with ``begin_op_log()`` and
``record_op_log=True``, records per (batch, group) lane its NEW_CLUSTER and JOIN rows;
``take_op_log()`` after every step must return the same rows and lengths here (atol = 0),
with recording leaving the flush unchanged.
"""
from __future__ import annotations

import os

import numpy as np
import pytest
import torch

from fixtures import CONFIGS, config, make_stream
from test_flush_gpu import make_cache, push_chunk

pytestmark = pytest.mark.gpu
HERE = os.path.dirname(os.path.abspath(__file__))


@pytest.mark.parametrize("name", [c["name"] for c in CONFIGS])
def test_op_log_matches_reference(name):
    cfg = config(name)
    stream = make_stream(cfg)
    ref = np.load(os.path.join(HERE, "golden", f"oplog_{name}.npz"))
    cache = make_cache(cfg, stream)
    cache.begin_op_log()
    for step, chunk in enumerate(stream["chunks"]):
        dt = cache.level_k.dtype
        k = torch.from_numpy(chunk["k"]).to("cuda", dt)
        kr = torch.from_numpy(chunk["k_raw"]).to("cuda", dt)
        v = torch.from_numpy(chunk["v"]).to("cuda", dt)
        pos = torch.from_numpy(chunk["pos"]).cuda() if chunk.get("pos") is not None else None
        cache.add_recent(k, v, k_raw=kr, input_pos=pos, span_ends=chunk["span_ends"].tolist(), record_op_log=True)
        log, lengths = cache.take_op_log()
        want_len = ref[f"step{step}/op_log_len"]
        np.testing.assert_array_equal(lengths.cpu().numpy(), want_len, err_msg=f"step {step} lengths")
        want = ref[f"step{step}/op_log"]
        got = log.cpu().numpy()
        assert got.shape == want.shape, (step, got.shape, want.shape)
        for b in range(want.shape[0]):
            for g in range(want.shape[1]):
                n = int(want_len[b, g])
                np.testing.assert_array_equal(got[b, g, :n], want[b, g, :n], err_msg=f"step {step} lane {(b, g)}")
        np.testing.assert_array_equal(cache.level_count.cpu().numpy(), ref[f"step{step}/level_count"])


def test_op_log_overflow_raises():
    cfg = config(CONFIGS[0]["name"])
    stream = make_stream(cfg)
    cache = make_cache(cfg, stream)
    cache.begin_op_log()
    cache.op_log = cache.op_log[:, :, :4].contiguous()   # far too small for one flush
    with pytest.raises(RuntimeError, match="overflow"):
        for chunk in stream["chunks"]:
            dt = cache.level_k.dtype
            k = torch.from_numpy(chunk["k"]).to("cuda", dt)
            kr = torch.from_numpy(chunk["k_raw"]).to("cuda", dt)
            v = torch.from_numpy(chunk["v"]).to("cuda", dt)
            pos = torch.from_numpy(chunk["pos"]).cuda() if chunk.get("pos") is not None else None
            cache.add_recent(k, v, k_raw=kr, input_pos=pos, span_ends=chunk["span_ends"].tolist(),
                             record_op_log=True)
            cache.take_op_log()


def test_op_log_replay_of_an_alpha_flush_raises_as_the_reference():
    """Outside an update-tape context the reference cannot replay an Alpha flush from an op-log
    (log_kv_cache.py:5060-5061): the chunk is appended, the flush raises, the window keeps the
    chunk.  Chunks that flush nothing pass."""
    cfg = config(CONFIGS[0]["name"])
    stream = make_stream(cfg)
    cache = make_cache(cfg, stream)
    log = torch.zeros(cfg["batch"], cfg["groups"], 4, 4, dtype=torch.int32, device="cuda")
    length = torch.zeros(cfg["batch"], cfg["groups"], dtype=torch.int32, device="cuda")
    dt = cache.level_k.dtype
    raised = False
    for chunk in stream["chunks"][:3]:
        k = torch.from_numpy(chunk["k"]).to("cuda", dt)
        kr = torch.from_numpy(chunk["k_raw"]).to("cuda", dt)
        v = torch.from_numpy(chunk["v"]).to("cuda", dt)
        before = cache.recent_count
        try:
            cache.add_recent(k, v, k_raw=kr, span_ends=chunk["span_ends"].tolist(), replay_op_log=log,
                             replay_op_log_len=length)
        except RuntimeError as exc:
            assert "AlphaLogKV replay requires semantic_replay_updates" in str(exc)
            assert cache.recent_count == before + k.size(2)
            raised = True
            break
    assert raised
