"""Route overlap: flush decisions on a side stream beside the caller's queued work.

The reference's ``LOGKV_ROUTE_OVERLAP`` (litgpt/log_kv_cache.py:3814-3849) moves the route
decisions of a flush onto a high-priority side stream ordered only after the previous flush,
and returns the commit to the caller's stream; results are unchanged.  Here every golden stream
runs twice, once plainly and once with overlap while the caller's stream is kept busy (a GPU
sleep queued before each chunk), and every device buffer must be equal after every step; one
more case shows that the decisions really complete while the caller's stream is still busy.
"""
from __future__ import annotations

import pytest
import torch

from fixtures import CONFIGS, config, make_stream
from test_flush_gpu import make_cache
from test_update_tape_gpu import assert_state, push, state

pytestmark = pytest.mark.gpu
BUSY_CYCLES = 2_000_000  # about a millisecond of the caller's stream per chunk


@pytest.mark.parametrize("name", [c["name"] for c in CONFIGS])
def test_overlapped_flushes_equal_plain_flushes(name):
    cfg = config(name)
    stream = make_stream(cfg)
    plain, over = make_cache(cfg, stream), make_cache(cfg, stream)
    over._route_overlap = True
    flushes = 0
    with torch.no_grad():
        for chunk in stream["chunks"]:
            push(plain, cfg, chunk, record_op_log=True)
            torch.cuda._sleep(BUSY_CYCLES)
            before = over._flush_cursor
            push(over, cfg, chunk, record_op_log=True)
            flushes += over._flush_cursor - before
            assert over.read_status() == 0
            assert_state(over, state(plain))
            got, want = over.take_op_log(), plain.take_op_log()
            if want[0] is None:
                assert got[0] is None and got[1] is None
            else:
                assert torch.equal(got[1], want[1]) and torch.equal(got[0], want[0])
    assert flushes > 1


def test_decisions_finish_while_the_callers_stream_is_busy():
    from test_flush_gpu import torch_dtype
    cfg = next(c for c in CONFIGS if c["beta"])
    stream = make_stream(cfg)
    cache = make_cache(cfg, stream)
    cache._route_overlap = True
    chunks = iter(stream["chunks"])
    dt = torch_dtype(cfg)
    with torch.no_grad():
        while cache._route_ready is None:          # up to and including the first flush
            push(cache, cfg, next(chunks))
        overlapped = False
        for chunk in chunks:
            # Inputs on the device first: a pageable upload would wait behind the sleep.
            k, kr, v = (torch.from_numpy(chunk[n]).to("cuda", dt) for n in ("k", "k_raw", "v"))
            pos = torch.from_numpy(chunk["pos"]).cuda() if chunk.get("pos") is not None else None
            ends = torch.from_numpy(chunk["span_ends"].astype("uint8")).cuda()
            torch.cuda.synchronize()
            rows = cache._route_ready_rows
            torch.cuda._sleep(400_000_000)          # a few hundred milliseconds
            before = cache._flush_cursor
            cache.add_recent(k, v, k_raw=kr, input_pos=pos, span_ends=chunk["span_ends"].tolist(),
                             span_ends_device=ends)
            if cache._flush_cursor > before and rows >= cfg["granularity"]:
                cache._route_done.synchronize()     # the decisions, on the side stream
                overlapped = not torch.cuda.current_stream().query()
                torch.cuda.synchronize()
                break
            torch.cuda.synchronize()
    assert overlapped, "decisions waited for the caller's stream"


def test_overlap_under_graph_capture_matches_plain_flushes():
    """Flushes captured in CUDA graphs with overlap on: a flush whose previous flush ran in
    another capture (or eagerly) does not fork; two flushes in one capture fork within it.
    Each graph is replayed once, in order; every buffer equals the plain eager cache's."""
    from test_flush_gpu import torch_dtype
    cfg = next(c for c in CONFIGS if c["beta"] and c["chunk"] == c["granularity"])
    stream = make_stream(cfg)
    plain, over = make_cache(cfg, stream), make_cache(cfg, stream)
    over._route_overlap = True
    dt = torch_dtype(cfg)
    chunks = stream["chunks"]
    with torch.no_grad():
        for chunk in chunks[:2]:                       # fill the window, first flush (eager)
            push(plain, cfg, chunk)
            push(over, cfg, chunk)
        groups = [chunks[2:3], chunks[3:5]]            # one flush alone, then two in one capture
        for group in groups:
            staged = []
            for chunk in group:
                push(plain, cfg, chunk)
                staged.append(tuple(torch.from_numpy(chunk[n]).to("cuda", dt) for n in ("k", "k_raw", "v"))
                              + (torch.from_numpy(chunk["span_ends"].astype("uint8")).cuda(),
                                 chunk["span_ends"].tolist()))
            torch.cuda.synchronize()
            graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(graph):
                for k, kr, v, ends, ends_host in staged:
                    over.add_recent(k, v, k_raw=kr, span_ends=ends_host, span_ends_device=ends)
            graph.replay()
            torch.cuda.synchronize()
            assert over.read_status() == 0
            assert_state(over, state(plain))
            del graph
