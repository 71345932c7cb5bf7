"""Update tape: record every flush of a golden stream, then replay the records.

Mirrors the reference's tests/test_log_kv_update_replay.py (record under
``_semantic_update_context(tape)``, reset, replay under ``replay=True`` without
rerouting, state equal after every step at atol=0; missing and out-of-order
records raise; replay onto a prefilled cache).  Here the records are device
buffers written by ``logkv_flush_record`` and applied by ``logkv_flush_replay``.
"""
from __future__ import annotations

from unittest.mock import patch

import pytest
import torch

from fixtures import CONFIGS, config, make_stream
from test_flush_gpu import make_cache, push_chunk, torch_dtype

pytestmark = pytest.mark.gpu


def state(cache):
    """Every device buffer of the cache (named and private), cloned."""
    out = {name: x.clone() for name, x in cache.named_buffers()}
    for name in ("_span_len", "_span_closed", "_span_count", "_row_count", "_alpha_count_dev", "_recent_ends"):
        out[name] = getattr(cache, name).clone()
    return out


def assert_state(cache, expected, skip=()):
    for name, x in state(cache).items():
        if name in skip:
            continue
        assert torch.equal(x, expected[name]), name


def push(cache, cfg, chunk, **kw):
    dt = torch_dtype(cfg)
    k = torch.from_numpy(chunk["k"]).to("cuda", dt)
    kr = torch.from_numpy(chunk["k_raw"]).to("cuda", dt)
    v = torch.from_numpy(chunk["v"]).to("cuda", dt)
    pos = torch.from_numpy(chunk["pos"]).cuda() if chunk.get("pos") is not None else None
    cache.add_recent(k, v, k_raw=kr, input_pos=pos, span_ends=chunk["span_ends"].tolist(), **kw)


@pytest.mark.parametrize("name", [c["name"] for c in CONFIGS])
def test_replay_restores_every_step_without_routing(name):
    from logkv_b200 import _SemanticReplayUpdates
    cfg = config(name)
    stream = make_stream(cfg)
    cache = make_cache(cfg, stream)
    tape = _SemanticReplayUpdates()
    expected = []
    with torch.no_grad(), cache._semantic_update_context(tape):
        for chunk in stream["chunks"]:
            push(cache, cfg, chunk, record_op_log=True)
            expected.append(state(cache))
    assert tape.tensors and cache._active_updates is None and cache._update_actions is None
    for _ in range(2):
        cache.reset_parameters()
        with patch.object(cache, "flush_device", side_effect=AssertionError("rerouted")):
            for chunk, want in zip(stream["chunks"], expected):
                with torch.no_grad(), cache._semantic_update_context(tape, replay=True):
                    push(cache, cfg, chunk)
                assert cache.read_status() == 0
                assert_state(cache, want)
    assert cache._active_updates is None and not cache._replaying_updates


def test_replay_uses_recorded_payload_and_decisions():
    """Changed inputs at replay: the flushed rows, decisions and cuts are the recorded ones;
    only the window rows that stay in the window follow the new inputs."""
    from logkv_b200 import _SemanticReplayUpdates
    cfg = next(c for c in CONFIGS if c["beta"] and c["dtype"] == "bf16")
    stream = make_stream(cfg)
    cache = make_cache(cfg, stream)
    tape = _SemanticReplayUpdates()
    expected = []
    with torch.no_grad(), cache._semantic_update_context(tape):
        for chunk in stream["chunks"]:
            push(cache, cfg, chunk, record_op_log=True)
            expected.append(state(cache))
    cache.reset_parameters()
    window = {"recent_k", "recent_k_raw", "recent_v"}
    for chunk, want in zip(stream["chunks"], expected):
        changed = dict(chunk, k=chunk["k"] * 10, k_raw=chunk["k_raw"] * 10, v=chunk["v"] * -7)
        with torch.no_grad(), cache._semantic_update_context(tape, replay=True):
            push(cache, cfg, changed)
        assert_state(cache, want, skip=window)


def test_replay_errors_and_prefilled_cache():
    from logkv_b200 import _SemanticReplayUpdates
    cfg = next(c for c in CONFIGS if c["beta"])
    stream = make_stream(cfg)
    chunks = stream["chunks"]
    a, b = make_cache(cfg, stream), make_cache(cfg, stream)
    # Prefill both the same way (no recording) up to and including the first flush.
    first_flush = None
    for i, chunk in enumerate(chunks):
        before = a._flush_cursor
        push(a, cfg, chunk)
        push(b, cfg, chunk)
        if a._flush_cursor > before:
            first_flush = i
            break
    assert first_flush is not None
    tape = _SemanticReplayUpdates()
    rest = chunks[first_flush + 1:]
    with torch.no_grad(), a._semantic_update_context(tape):
        for chunk in rest:
            push(a, cfg, chunk, record_op_log=True)
    with torch.no_grad(), b._semantic_update_context(tape, replay=True):
        for chunk in rest:
            push(b, cfg, chunk)
    assert_state(b, state(a))
    # The same records cannot be applied again at later cursors.
    with b._semantic_update_context(tape, replay=True), pytest.raises(RuntimeError, match="out of order"):
        for chunk in rest:
            push(b, cfg, chunk)
    # No record at all: replay refuses to reroute.
    fresh = make_cache(cfg, stream)
    with fresh._semantic_update_context(_SemanticReplayUpdates(), replay=True), \
            pytest.raises(RuntimeError, match="missing"):
        for chunk in chunks:
            push(fresh, cfg, chunk)
    # Recording needs record_op_log=True; outside a context, an op-log cannot replay an Alpha flush
    # (the reference's error, log_kv_cache.py:5060-5061, raised when the chunk flushes).
    fresh.reset_parameters()
    with fresh._semantic_update_context(_SemanticReplayUpdates()), pytest.raises(RuntimeError, match="record_op_log"):
        for chunk in chunks:
            push(fresh, cfg, chunk)
    fresh.reset_parameters()
    with pytest.raises(RuntimeError, match="AlphaLogKV replay requires semantic_replay_updates"):
        for chunk in chunks:
            push(fresh, cfg, chunk, replay_op_log=torch.zeros(1))
