"""Benchmark of the SemanticLogKV flush path on B200 (driver contract: one JSON line on rank 0).

Workload (Qwen3-0.6B-shaped streaming prefill): 28 layer
caches of 8 KV groups x head dim 128 (bf16), a 32768-token stream in 2048-token
chunks, K=12 clusters, B=128 slots (B'=125 after the exact pool), recent window
2048, flush granularity 2048, exact pool 256 tokens with 64-token spans, Beta on,
mid anchors.  One step = the whole stream through all 28 layers: 16 add_recent
calls per layer, 15 of which flush 2048 tokens (420 flushes per step), starting
from empty caches.  Keys are synthetic (a seeded 12-component Gaussian mixture
per layer and group with 5% far orphans; the model's projections are not part of
the path); span boundaries every 23rd token.

value     = device time per flush (chunk x layer), us, CUDA-graph replay of whole
            steps with inputs resident in HBM (each step's 5.6 GB of chunk inputs is
            larger than L2).  Layer l's add_recent calls run on stream l % --streams
            (default 28): the layers' caches are independent, so their flushes overlap,
            while each layer's chunks stay in order on its stream.
e2e       = the same metric through the public API: add_recent called eagerly per
            chunk and layer on the layers' streams, with every chunk's K, pre-RoPE K, V
            and span-end flags copied from pinned host memory inside the timed region
            and every layer's alpha_count read back.
roofline  = the ladder cascade kernel (the dominant flush stage): algorithmic
            bytes of its rows (549 B per bf16 row: K and V 256 B each, w 4 B,
            p_lo/p_hi/sum_wp/order 8 B each, pad 1 B) over its CUDA-event time,
            against the measured HBM copy bandwidth.
Other legs on the same line: decode (configs[3], with and without committing
generated tokens), prefill chunk attention, flush-and-attend, kv_sharded
(configs[2]), unified (configs[4]: unified-route flushes of 32 streams x 8 groups
per rank), and the reference's own CPU timings of configs[0] and of the unified
flush, recorded in the build container (tests/golden/*_timing.json).
--impl reference times the CPU oracle port (a numpy restatement of the
reference's flush) on every host core: one worker process per layer, --warmup
untimed and --steps timed steps, a step being one flush in every worker.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

WORKLOAD = dict(workload="qwen3-0.6b streaming prefill flush (28 layers, 32K tokens, 2048-token flushes)",
                layers=28, groups=8, head_dim=128, clusters=12, B=128, recent=2048, granularity=2048,
                exact=256, span_cap=64, beta=True, tokens=32768, chunk=2048, batch_per_rank=1, dtype="bf16")
ROW_BYTES = 256 + 256 + 4 + 4 * 8 + 1   # one bf16 ladder entry (13 fields, first-order subset)
# DRAM bytes (dram__bytes_read.sum + dram__bytes_write.sum) of one flush's cascade kernels (merge
# and move) in the one-launch ncu capture of this build at this layer shape (the
# profiling command is in the cascade profile summary).  Written rows mostly stay in L2 within the
# launch, so the figure is below the algorithmic bytes.
CASCADE_TRAFFIC = 15_832_832 + 0 + 20_753_408 + 2_816
# The same for one chunk attention launch (chunk_attn_tc_kernel, the prefill leg's shape).
PREFILL_TRAFFIC = 51_042_816 + 705_536
FLUSH_KERNELS = 12                      # kernel launches per flushing layer-chunk (the last writes the chunk)
METRIC = "flush us per 2048-tok chunk/layer"


def measured_peaks(key: str = "hbm_gbs"):
    """(peak, "measured" | "fallback"): HBM copy GB/s or burst bf16 GEMM TFLOP/s of this pool's B200s."""
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(path):
        with open(path) as fh:
            d = json.load(fh)
        return float(d[key]), "measured"
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0}[key], "fallback"


class ClockSampler:
    """nvidia-smi samples of SM clock and throttle reasons during the timed region."""

    def __init__(self, index: int):
        self.index, self.samples, self.proc = index, [], None

    def __enter__(self):
        q = ("clocks.sm,clocks.max.sm,clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
        try:
            self.proc = subprocess.Popen(["nvidia-smi", "-i", str(self.index), f"--query-gpu={q}",
                                          "--format=csv,noheader,nounits", "-lms", "100"],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.thread = threading.Thread(target=self._read, daemon=True)
            self.thread.start()
        except (OSError, FileNotFoundError):
            self.proc = None
            return self
        # nvidia-smi takes a moment to start: wait for its first sample so that a short timed
        # region is still covered.
        t0 = time.time()
        while not self.samples and time.time() - t0 < 5.0 and self.proc.poll() is None:
            time.sleep(0.01)
        self.n_start = len(self.samples)
        return self

    def _read(self):
        for line in self.proc.stdout:
            parts = [p.strip() for p in line.split(",")]
            if len(parts) == 6:
                self.samples.append(parts)

    def __exit__(self, *exc):
        if self.proc:
            # one more sample at the end of the region (at most one sampling period away)
            t0 = time.time()
            while len(self.samples) <= getattr(self, "n_start", 0) and time.time() - t0 < 1.0:
                time.sleep(0.01)
            self.proc.terminate()
            self.proc.wait(timeout=5)

    def summary(self):
        if not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        sm = [float(s[0]) for s in self.samples if s[0].replace(".", "").isdigit()]
        mx = [float(s[1]) for s in self.samples if s[1].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for s in self.samples for i in range(4) if s[2 + i].lower() == "active"})
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": reasons, "samples": len(self.samples)}


# ---------------------------------------------------------------------------------------------- inputs
def make_inputs(torch, cfg, device, seed):
    """Per layer and chunk: k_raw, post-RoPE k and v (bf16, on device), plus the span-end table."""
    from logkv_b200.workload import rope_tables
    G, D, K, T, n_chunks = cfg["groups"], cfg["head_dim"], cfg["clusters"], cfg["chunk"], cfg["tokens"] // cfg["chunk"]
    gen = torch.Generator(device=device).manual_seed(seed)
    cos_np, sin_np = rope_tables(cfg["tokens"], D, base=1e6)
    cos = torch.from_numpy(cos_np).to(device)
    sin = torch.from_numpy(sin_np).to(device)
    ends_row = [(i % 23) == 22 for i in range(T)]
    ends_dev = torch.tensor([ends_row], dtype=torch.uint8, device=device)
    layers = []
    N = n_chunks
    pos = torch.arange(N * T, device=device).view(N, 1, T)
    for layer in range(cfg["layers"]):
        # All chunks of one layer at once (few launches); chunk c is the view [c:c+1].
        centres = torch.randn(G, K, D, generator=gen, device=device)
        z = torch.randint(0, K, (N, G, T), generator=gen, device=device)
        base = centres[torch.arange(G, device=device)[None, :, None], z]
        noise = torch.randn(N, G, T, D, generator=gen, device=device) * 0.3
        orphan = torch.rand(N, G, T, generator=gen, device=device) < 0.05
        u = torch.randn(N, G, T, D, generator=gen, device=device)
        u = u / u.norm(dim=-1, keepdim=True) * (4 * 0.3 * D ** 0.5)
        kr = torch.where(orphan[..., None], base + u, base + noise)
        half = D // 2
        rot = torch.cat([-kr[..., half:], kr[..., :half]], dim=-1)
        k = (kr * cos[pos] + rot * sin[pos]).bfloat16()
        v = torch.randn(N, G, T, D, generator=gen, device=device).bfloat16()
        kr = kr.bfloat16()
        del base, noise, u, rot
        layers.append([(k[c:c + 1], kr[c:c + 1], v[c:c + 1]) for c in range(N)])
    return layers, cos, sin, [ends_row], ends_dev


def make_caches(torch, cfg, device, cos, sin):
    from logkv_b200.cache import LogStructuredKVCache
    caches = []
    for _ in range(cfg["layers"]):
        caches.append(LogStructuredKVCache(
            (cfg["batch_per_rank"], cfg["groups"], cfg["tokens"], cfg["head_dim"]),
            (cfg["batch_per_rank"], cfg["groups"], cfg["tokens"], cfg["head_dim"]),
            B=cfg["B"], recent_size=cfg["recent"], device=device, dtype=torch.bfloat16,
            semantic_clusters=True, semantic_anchor_mode="mid", allocate_second_order=False,
            cluster_k_max=cfg["clusters"], semantic_flush_granularity=cfg["granularity"],
            semantic_centroid_backend="parallel", semantic_replay_updates=True,
            alpha_exact_tokens=cfg["exact"], alpha_span_max_tokens=cfg["span_cap"],
            beta_novelty=cfg["beta"], beta_adaptive_merge=cfg["beta"], cos_cache=cos, sin_cache=sin,
            rope_n_elem=cfg["head_dim"]))
    return caches


def run_step(caches, layers, ends_host, ends_dev=None, streams=None):
    """One step: every layer's chunks in chunk-major order.

    With ``streams``, layer l's cache is updated on ``streams[l % S]``: the layers' caches are
    independent, so their flushes overlap (as in a model's prefill, where layer l's flush only
    has to finish before layer l's next chunk).  The streams fork from and join back into the
    current stream, so the step can be captured in one CUDA graph.
    """
    import torch
    n_chunks = len(layers[0])
    if not streams:
        for cache in caches:
            cache.reset_parameters()
        for c in range(n_chunks):
            for cache, chunks in zip(caches, layers):
                k, kr, v = chunks[c]
                cache.add_recent(k, v, k_raw=kr, span_ends=ends_host, span_ends_device=ends_dev)
        return
    main = torch.cuda.current_stream()
    for st in streams:
        st.wait_stream(main)
    for li, cache in enumerate(caches):
        with torch.cuda.stream(streams[li % len(streams)]):
            cache.reset_parameters()
    for c in range(n_chunks):
        for li, (cache, chunks) in enumerate(zip(caches, layers)):
            k, kr, v = chunks[c]
            with torch.cuda.stream(streams[li % len(streams)]):
                cache.add_recent(k, v, k_raw=kr, span_ends=ends_host, span_ends_device=ends_dev)
    for st in streams:
        main.wait_stream(st)


# ---------------------------------------------------------------------------------------------- our arm
def bench_ours(args, rank, world, local_rank):
    import torch
    import torch.distributed as dist
    device = torch.device("cuda", local_rank)
    torch.cuda.set_device(device)
    cfg = dict(WORKLOAD)
    cfg["layers"] = args.layers
    layers, cos, sin, ends_host, ends_dev = make_inputs(torch, cfg, device, seed=1234 + rank)
    caches = make_caches(torch, cfg, device, cos, sin)
    flushes_per_step = cfg["layers"] * (cfg["tokens"] // cfg["chunk"] - cfg["recent"] // cfg["chunk"])
    stream = torch.cuda.Stream(device)
    torch.cuda.synchronize()   # inputs were written on the default stream
    streams = [torch.cuda.Stream(device) for _ in range(args.streams)] if args.streams > 1 else None
    # Warm-up (eager), then one CUDA graph per step.
    with torch.cuda.stream(stream):
        for _ in range(args.warmup):
            run_step(caches, layers, ends_host, ends_dev, streams)
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=stream):
        run_step(caches, layers, ends_host, ends_dev, streams)
    with torch.cuda.stream(stream):
        for _ in range(max(1, args.warmup)):
            graph.replay()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local_rank) as clocks:
        torch.cuda.synchronize()
        with torch.cuda.stream(stream):
            start.record(stream)
            for _ in range(args.steps):
                graph.replay()
            stop.record(stream)
        torch.cuda.synchronize()
    ms = start.elapsed_time(stop)
    if world > 1:
        t = torch.tensor([ms], device=device)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    us_per_flush = ms * 1000.0 / (args.steps * flushes_per_step)
    ms_per_step = ms / args.steps

    # Per-stage profile (eager, one step): stage events around every flush.
    from logkv_b200._lib import FLUSH_STAGES
    nstage = len(FLUSH_STAGES)
    events = [[torch.cuda.Event(enable_timing=True) for _ in range(nstage + 1)] for _ in range(flushes_per_step)]
    for evs in events:
        for e in evs:
            e.record(stream)
    torch.cuda.synchronize()
    before = [c.read_counters() for c in caches]
    stage_ms = [0.0] * nstage
    with torch.cuda.stream(stream):
        for cache in caches:
            cache.reset_parameters()
        idx = 0
        for c in range(len(layers[0])):
            for cache, chunks in zip(caches, layers):
                k, kr, v = chunks[c]
                will_flush = cache.recent_count + k.size(2) > cache.recent_size
                cache.profile_events = events[idx] if will_flush else None
                cache.add_recent(k, v, k_raw=kr, span_ends=ends_host, span_ends_device=ends_dev)
                idx += 1 if will_flush else 0
                cache.profile_events = None
    torch.cuda.synchronize()
    per_flush = [[] for _ in range(nstage)]
    for evs in events:
        for i in range(nstage):
            t = evs[i].elapsed_time(evs[i + 1])
            stage_ms[i] += t
            per_flush[i].append(t)
    after = [c.read_counters() for c in caches]
    delta = {k: sum(a[k] - b[k] for a, b in zip(after, before)) for k in after[0]}
    stages_us = {name: round(stage_ms[i] * 1000.0 / flushes_per_step, 2) for i, name in enumerate(FLUSH_STAGES)}
    stages_med = {name: round(statistics.median(per_flush[i]) * 1000.0, 2) for i, name in enumerate(FLUSH_STAGES)}
    stages_max = {name: round(max(per_flush[i]) * 1000.0, 2) for i, name in enumerate(FLUSH_STAGES)}
    # Algorithmic cascade bytes: rows read and written by the ladder append, carries excluded
    # (a carried row is produced and consumed inside the cascade).
    casc_rows = delta["storage_read"] + delta["stage_read"] + delta["survivor"] + delta["fill"] + delta["clear"]
    casc_bytes_per_launch = casc_rows * ROW_BYTES / flushes_per_step
    casc_bytes_carry = (casc_rows + delta["carry"]) * ROW_BYTES / flushes_per_step
    casc_s = stage_ms[FLUSH_STAGES.index("cascade")] / 1000.0 / flushes_per_step
    peak, peak_kind = measured_peaks()
    achieved = casc_bytes_per_launch / casc_s / 1e9
    # Whole-flush algorithmic bytes (ladder rows + Alpha/route reads of [pool|flush] K,V + pool rewrite).
    e = 2
    P, F, G, D = cfg["exact"], cfg["granularity"], cfg["groups"], cfg["head_dim"]
    flush_rows = delta["storage_read"] + delta["stage_read"] + delta["survivor"] + delta["fill"] + delta["clear"]
    flush_bytes = flush_rows * ROW_BYTES / flushes_per_step + (P + F) * G * D * 2 * e + P * G * D * 2 * e
    flush_achieved = flush_bytes / (us_per_flush * 1e-6) / 1e9

    # e2e: public API, eager, host inputs copied each chunk.
    host = []
    ends_pinned = ends_dev.cpu().pin_memory()
    for chunks in layers:
        host.append([tuple(t[:, :, :].cpu().pin_memory() for t in chunks[c]) + (ends_pinned,) for c in range(2)])
    # A ring of device slots; a copy stream fills slot n % nslot with layer-chunk n's inputs
    # (k, k_raw, v and the span-end flags) while earlier layer-chunks are flushed on their
    # layers' streams (events order each slot's reuse).
    nslot = 2 * max(1, args.streams)
    dev_buf = [tuple(torch.empty_like(t, device=device) for t in host[0][0]) for _ in range(nslot)]
    copy_stream = torch.cuda.Stream(device)
    torch.cuda.synchronize()   # inputs were written on the default stream
    filled = [torch.cuda.Event() for _ in range(nslot)]
    consumed = [torch.cuda.Event() for _ in range(nslot)]
    h2d_per_step = sum(t.numel() * t.element_size() for t in host[0][0]) * len(layers) * len(layers[0])
    lstreams = streams or [stream]
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    e_start, e_stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e_start.record(stream)
    copy_stream.wait_stream(stream)
    for st in lstreams:
        st.wait_stream(stream)
    n = 0
    for _ in range(args.steps):
        for li, cache in enumerate(caches):
            with torch.cuda.stream(lstreams[li % len(lstreams)]):
                cache.reset_parameters()
        for c in range(len(layers[0])):
            for li, cache in enumerate(caches):
                slot = n % nslot
                buf = dev_buf[slot]
                ls = lstreams[li % len(lstreams)]
                with torch.cuda.stream(copy_stream):
                    if n >= nslot:
                        copy_stream.wait_event(consumed[slot])
                    for d, h in zip(buf, host[li][c % 2]):
                        d.copy_(h, non_blocking=True)
                    filled[slot].record(copy_stream)
                with torch.cuda.stream(ls):
                    ls.wait_event(filled[slot])
                    cache.add_recent(buf[0], buf[2], k_raw=buf[1], span_ends=ends_host, span_ends_device=buf[3])
                    consumed[slot].record(ls)
                n += 1
        for st in lstreams:
            stream.wait_stream(st)
        with torch.cuda.stream(stream):
            readback = torch.stack([cache._alpha_count_dev for cache in caches]).to("cpu", non_blocking=False)
        for st in lstreams:
            st.wait_stream(stream)
    e_stop.record(stream)
    torch.cuda.synchronize()
    e_ms = e_start.elapsed_time(e_stop)
    if world > 1:
        t = torch.tensor([e_ms], device=device)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        e_ms = float(t.item())
    e2e_us = e_ms * 1000.0 / (args.steps * flushes_per_step)
    del readback
    chunks_per_step = cfg["layers"] * (cfg["tokens"] // cfg["chunk"])
    n_launch = (flushes_per_step * FLUSH_KERNELS + (chunks_per_step - flushes_per_step)) * args.steps
    return dict(value=us_per_flush * 1.0 / world, ms_per_step=ms_per_step, e2e_us=e2e_us / world,
                h2d=h2d_per_step * world, stages=stages_us, stages_med=stages_med, stages_max=stages_max,
                counters=delta, flushes_per_step=flushes_per_step,
                roofline={"bound": "hbm", "kernel": "ladder cascade (cascade_merge_kernel + cascade_move_kernel)",
                          "achieved": round(achieved, 1), "peak": peak, "peak_kind": peak_kind, "unit": "GB/s",
                          "frac": round(achieved / peak, 4), "traffic": CASCADE_TRAFFIC,
                          "traffic_source": "ncu capture of this build's cascade kernels, one flush, same layer shape",
                          "bytes_per_launch": round(casc_bytes_per_launch),
                          "bytes_per_launch_with_carries": round(casc_bytes_carry),
                          "frac_with_carries": round(casc_bytes_carry / casc_s / 1e9 / peak, 4),
                          "launch_us": round(casc_s * 1e6, 2)},
                flush_roofline={"achieved": round(flush_achieved, 1), "unit": "GB/s",
                                "frac": round(flush_achieved / peak, 4), "bytes_per_flush": round(flush_bytes)},
                clocks=clocks.summary(), launches=n_launch, inputs=(caches, layers, ends_host, ends_dev))


def bench_flush_attend(args, rank, world, local_rank, inputs):
    """Flush-and-attend prefill in model order: per layer-chunk the chunk attention of the layer's
    16 query heads over its cache, then ``add_recent`` of the chunk (a 2048-token flush); chunks
    in sequence, the 28 layers in sequence within a chunk, on one stream, one CUDA graph per step.
    Timed three ways: with the route decisions on the caller's stream; with route overlap (the
    decisions of each flush on a side stream, ordered only after the layer's previous flush); and
    with route overlap and each layer's ``add_recent`` on that layer's own stream, ordered after
    the layer's attention, with the layer's next attention ordered after it (a layer's flush only
    has to finish before that layer's next chunk, so it runs beside the next layers' attention).
    """
    import torch
    import torch.distributed as dist
    from logkv_b200.attention import log_kv_chunk_attention
    caches, layers, ends_host, ends_dev = inputs
    device = caches[0].level_k.device
    H, D, T = 16, WORKLOAD["head_dim"], WORKLOAD["chunk"]
    gen = torch.Generator(device=device).manual_seed(77 + rank)
    q = torch.randn(1, H, T, D, generator=gen, device=device).to(torch.bfloat16)
    out = torch.empty_like(q)
    scale = D ** -0.5
    stream = torch.cuda.Stream(device)
    torch.cuda.synchronize()   # inputs were written on the default stream
    lstreams = [torch.cuda.Stream(device) for _ in caches]
    n_chunks = len(layers[0])

    def step(layer_streams):
        main = torch.cuda.current_stream()
        if layer_streams:
            for st in lstreams:
                st.wait_stream(main)                      # fork (joins a capture too)
        for cache in caches:
            cache.reset_parameters()
        for c in range(n_chunks):
            for li, (cache, chunks) in enumerate(zip(caches, layers)):
                k, kr, v = chunks[c]
                if layer_streams:
                    main.wait_stream(lstreams[li])        # the layer's previous flush
                log_kv_chunk_attention(cache, q, k, v, scale, 0.0, out=out)
                if layer_streams:
                    lstreams[li].wait_stream(main)        # after this attention
                    with torch.cuda.stream(lstreams[li]):
                        cache.add_recent(k, v, k_raw=kr, span_ends=ends_host, span_ends_device=ends_dev)
                else:
                    cache.add_recent(k, v, k_raw=kr, span_ends=ends_host, span_ends_device=ends_dev)
        if layer_streams:
            for st in lstreams:
                main.wait_stream(st)

    us = {}
    for mode in ("plain", "overlap", "layer_streams"):
        overlap, layered = mode != "plain", mode == "layer_streams"
        for cache in caches:
            cache._route_overlap = overlap
        with torch.no_grad(), torch.cuda.stream(stream):
            for _ in range(max(1, args.warmup)):
                step(layered)
            torch.cuda.synchronize()
            graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(graph, stream=stream):
                step(layered)
            graph.replay()
            torch.cuda.synchronize()
            if world > 1:
                dist.barrier()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(stream)
            for _ in range(args.steps):
                graph.replay()
            e1.record(stream)
            torch.cuda.synchronize()
        del graph
        t = torch.tensor([e0.elapsed_time(e1)], device=device)
        if world > 1:
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
        us[mode] = round(t.item() * 1000.0 / (args.steps * n_chunks * len(caches)), 2)
    for cache in caches:
        cache._route_overlap = False
    return {"metric": "flush-and-attend prefill us per 2048-token chunk/layer (chunk attention + add_recent)",
            "unit": "us", "value": us["layer_streams"], "value_route_overlap_one_stream": us["overlap"],
            "value_one_stream": us["plain"],
            "config": {"layers": len(caches), "chunks": n_chunks, "heads": H, "groups": WORKLOAD["groups"],
                       "head_dim": D, "chunk": T, "flushes_per_step": len(caches) * (n_chunks - 1)}}


# ---------------------------------------------------------------------------------------------- unified route
UNIFIED = dict(workload="unified (Ward / radius) route flush, BASELINE configs[4]: 256 streams of 65536 tokens "
                        "batch-sharded over 8 ranks (32 per rank), 8 KV groups, head dim 128, bf16 K/V, K=12, B=128, "
                        "recent 2048 flushed 2048 at a time, exact pool 256 (span cap 64), Beta on; keys from a "
                        "48-component mixture per stream and group (sigma ~ U[0.1, 0.6], 10% orphans)",
               streams_per_rank=32, groups=8, head_dim=128, clusters=12, B=128, recent=2048, granularity=2048,
               exact=256, span_cap=64, max_seq=65536, components=48, orphan_frac=0.10)


def unified_reference_timing():
    """The reference's own CPU unified flush at this shape, timed in the build container
    (tests/golden/time_unified_reference.py writes tests/golden/unified_timing.json)."""
    path = os.path.join(ROOT, "tests", "golden", "unified_timing.json")
    if not os.path.exists(path):
        return None
    with open(path) as fh:
        t = json.load(fh)
    return {"s_per_stream_flush": round(statistics.median(t["flush_s"]), 3), "threads": t["threads"],
            "flushes": len(t["flush_s"]), "where": "build container CPU (the reference is not on the GPU box)",
            "kind": "reference"}


def configs0_reference_timing():
    """the reference's own CPU Torch flush (single layer, B=1, G=8, D=128, K=12,
    one 2048-token flush, planted spans; s_h = 1 / 12 / 32 and the 8-alive seeding case, fp32 and
    bf16), timed in the build container by tests/golden/make_fullshape.py (fullshape_timing.json)."""
    path = os.path.join(ROOT, "tests", "golden", "fullshape_timing.json")
    if not os.path.exists(path):
        return None
    with open(path) as fh:
        t = json.load(fh)
    per_case = {name: round(statistics.median(v["flush_s"]) * 1000.0, 1) for name, v in sorted(t.items())
                if "unified" not in name}
    return {"ms_per_flush_median_by_case": per_case,
            "ms_per_flush_median": round(statistics.median(per_case.values()), 1),
            "threads": next(iter(t.values()))["threads"], "kind": "reference",
            "where": "build container CPU (the reference is not on the GPU box)"}


def bench_unified(args, rank, world, local_rank):
    """Unified-route flushes of this rank's streams (batch-sharded: no collective).
    Chunk 0 fills each stream's window, --warmup flushes run untimed, then --steps flushes are timed
    with CUDA events around add_recent (inputs already on the device; each chunk is 2048 fresh
    tokens per stream).  Per-lane pass figures come from cache.read_unified()."""
    import torch
    import torch.distributed as dist
    from logkv_b200._lib import FLUSH_STAGES
    from logkv_b200.cache import LogStructuredKVCache
    from logkv_b200.workload import rope_tables
    cfg = UNIFIED | {"streams_per_rank": args.unified_streams}
    S, G, D, T = cfg["streams_per_rank"], cfg["groups"], cfg["head_dim"], cfg["granularity"]
    device = torch.device("cuda", local_rank)
    cos, sin = rope_tables(cfg["max_seq"] + 64, D)
    cache = LogStructuredKVCache(
        (S, G, cfg["max_seq"], D), (S, G, cfg["max_seq"], D), B=cfg["B"], recent_size=cfg["recent"], device=device,
        dtype=torch.bfloat16, semantic_clusters=True, cluster_k_max=cfg["clusters"], semantic_anchor_mode="mid",
        semantic_flush_granularity=T, allocate_second_order=False, alpha_exact_tokens=cfg["exact"],
        alpha_span_max_tokens=cfg["span_cap"], beta_novelty=True, beta_adaptive_merge=True,
        cos_cache=torch.from_numpy(cos), sin_cache=torch.from_numpy(sin), rope_n_elem=D, semantic_unified_route=True)
    gen = torch.Generator(device=device).manual_seed(7000 + rank)
    C = cfg["components"]
    centres = torch.randn(S, G, C, D, generator=gen, device=device)
    sigma = torch.rand(S, G, C, generator=gen, device=device) * 0.5 + 0.1
    si = torch.arange(S, device=device)[:, None, None]
    gi = torch.arange(G, device=device)[None, :, None]
    cos_d, sin_d = torch.from_numpy(cos).to(device), torch.from_numpy(sin).to(device)
    ends = (torch.arange(T) % 23 == 22).expand(S, T)
    ends_dev = ends.to(device, torch.uint8).contiguous()
    ends_host = ends.tolist()

    def chunk(c):
        z = torch.randint(0, C, (S, G, T), generator=gen, device=device)
        base, sig = centres[si, gi, z], sigma[si, gi, z][..., None]
        x = base + sig * torch.randn(S, G, T, D, generator=gen, device=device)
        u = torch.randn(S, G, T, D, generator=gen, device=device)
        u = u / u.norm(dim=-1, keepdim=True)
        orphan = torch.rand(S, G, T, generator=gen, device=device) < cfg["orphan_frac"]
        kr = torch.where(orphan[..., None], base + u * (4.0 * sig * D ** 0.5), x)
        pos = torch.arange(c * T, (c + 1) * T, device=device)
        half = D // 2
        rot = torch.cat([-kr[..., half:], kr[..., :half]], dim=-1)
        k = kr * cos_d[pos] + rot * sin_d[pos]
        v = torch.randn(S, G, T, D, generator=gen, device=device)
        return k.to(torch.bfloat16), kr.to(torch.bfloat16), v.to(torch.bfloat16)

    nstage = len(FLUSH_STAGES)
    stage_ms = [0.0] * nstage
    total_ms, figures = [], []
    warm = max(1, args.warmup)
    for c in range(1 + warm + args.steps):
        k, kr, v = chunk(c)
        timed = c > warm
        evs = [torch.cuda.Event(enable_timing=True) for _ in range(nstage + 1)] if timed else None
        for e in evs or []:
            e.record()
        torch.cuda.synchronize()
        cache.profile_events = evs
        cache.add_recent(k, v, k_raw=kr, span_ends=ends_host, span_ends_device=ends_dev)
        cache.profile_events = None
        torch.cuda.synchronize()
        if timed:
            total_ms.append(evs[0].elapsed_time(evs[-1]))
            for i in range(nstage):
                stage_ms[i] += evs[i].elapsed_time(evs[i + 1])
            figures.append(cache.read_unified())
    status = cache.read_status()
    t = torch.tensor([sum(total_ms) / len(total_ms)], device=device)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms = float(t.item())
    n = len(total_ms)
    route_ms = stage_ms[FLUSH_STAGES.index("seed_plan")] / n
    lanes = S * G
    mean = lambda key: round(float(sum(f[key].mean() for f in figures) / n), 1)  # noqa: E731
    rows_c = sum(float((f["cand_live"] + f["cand_merges"]).astype("float64").mean()) for f in figures) / n
    rows_g = mean("glob_rows")
    # Pair-matrix work per flush: every lane's two passes (upper-triangle Gram products, 2 flops each).
    gram_flop = lanes * D * (rows_c * (rows_c + 1) + rows_g * (rows_g + 1))
    dist_bytes = lanes * 4 * 2 * (rows_c ** 2 + rows_g ** 2)   # each matrix written once, read once by the first scan
    peak, kind = measured_peaks()
    ref = unified_reference_timing()
    out = {"metric": f"unified-route flush ms per 2048-token chunk of this rank's streams ({S} streams x {G} groups)",
           "unit": "ms", "value": round(ms, 3), "higher_is_better": False, "scaling": "weak",
           "tokens_per_s": round(S * world * T / (ms * 1e-3), 1),
           "us_per_lane_flush": round(ms * 1000.0 / lanes, 2), "status": status,
           "stages_ms": {name: round(stage_ms[i] / n, 3) for i, name in enumerate(FLUSH_STAGES)},
           "route_ms": round(route_ms, 3),
           "passes": {"candidate_rows": round(rows_c, 1), "candidate_rounds": mean("cand_rounds"),
                      "candidates": mean("candidates"), "global_rows": rows_g, "global_rounds": mean("glob_rounds"),
                      "ward_merges_per_flush": round(sum(float(f["ward_merges"].sum()) for f in figures) / n, 2)},
           "pair_matrix": {"gram_gflop_per_flush": round(gram_flop / 1e9, 2),
                           "dist_bytes_per_flush": int(dist_bytes),
                           "route_stage_dist_gbs": round(dist_bytes / (route_ms * 1e-3) / 1e9, 1),
                           "route_stage_dist_frac": round(dist_bytes / (route_ms * 1e-3) / 1e9 / peak, 4),
                           "peak_gbs": peak, "peak_kind": kind},
           "config": {k: v for k, v in cfg.items()} | {"flushes_timed": n, "ranks": world, "lanes_per_rank": lanes}}
    if ref is not None:
        out["cpu_reference"] = ref | {"ratio_per_stream": round(ref["s_per_stream_flush"] * 1000.0 / (ms / S), 1)}
    del cache
    torch.cuda.empty_cache()
    return out


# ---------------------------------------------------------------------------------------------- KV-head sharded
KVSHARD = dict(workload="qwen3-1.7b-shaped streaming prefill flush, one sequence KV-head-sharded "
                        "(BASELINE configs[2]: recent 4096, 2048-token flushes)",
               layers=28, groups=8, head_dim=128, clusters=12, B=128, recent=4096, granularity=2048,
               exact=256, span_cap=64, beta=True, tokens=32768, chunk=2048, batch_per_rank=1)


def bench_kv_sharded(args, rank, world, local_rank):
    """One long sequence, its 8 KV groups split over the ranks (G / world each).  Every chunk of
    the 28 layers is flushed through ``sharding.BatchedFlush``: each layer's score phase on its
    own stream, ONE all-gather of all layers' span parts per chunk (NCCL), then each layer's
    commit on its stream.  Timed two ways, whole steps captured in a CUDA graph, device time,
    max over ranks: the flushes alone (``value``, per layer-flush), and in model order
    (``flush_attend``, per layer-chunk): per layer the chunk attention of the rank's query heads
    over its cache and the all-gather of the attention outputs (``sharding.gather_heads``), then
    the layer's score phase on its stream, the chunk's one span-part exchange after the last
    layer, and the layers' commits beside the next chunk's attention."""
    import torch
    import torch.distributed as dist
    from logkv_b200.attention import log_kv_chunk_attention
    from logkv_b200.cache import LogStructuredKVCache
    from logkv_b200.sharding import BatchedFlush, gather_heads, group_block
    device = torch.device("cuda", local_rank)
    cfg = dict(KVSHARD)
    cfg["layers"] = args.kv_layers
    lo, hi = group_block(cfg["groups"], rank, world)
    layers, cos, sin, ends_host, ends_dev = make_inputs(torch, cfg, device, seed=4321)   # same on every rank
    layers = [[tuple(t[:, lo:hi].contiguous() for t in chunk) for chunk in chunks] for chunks in layers]
    group = dist.group.WORLD if world > 1 else None
    caches = [LogStructuredKVCache(
        (1, hi - lo, cfg["tokens"], cfg["head_dim"]), (1, hi - lo, cfg["tokens"], cfg["head_dim"]),
        B=cfg["B"], recent_size=cfg["recent"], device=device, dtype=torch.bfloat16, semantic_clusters=True,
        semantic_anchor_mode="mid", allocate_second_order=False, cluster_k_max=cfg["clusters"],
        semantic_flush_granularity=cfg["granularity"], semantic_centroid_backend="parallel",
        semantic_replay_updates=True, alpha_exact_tokens=cfg["exact"], alpha_span_max_tokens=cfg["span_cap"],
        beta_novelty=cfg["beta"], beta_adaptive_merge=cfg["beta"], cos_cache=cos, sin_cache=sin,
        rope_n_elem=cfg["head_dim"], kv_shard_group=group) for _ in range(cfg["layers"])]
    batch = BatchedFlush(caches, group)
    n_chunks = cfg["tokens"] // cfg["chunk"]
    flushes_per_step = cfg["layers"] * (n_chunks - cfg["recent"] // cfg["chunk"])
    H_local, D, T = 16 // cfg["groups"] * (hi - lo), cfg["head_dim"], cfg["chunk"]
    gen = torch.Generator(device=device).manual_seed(99 + rank)
    q = torch.randn(1, H_local, T, D, generator=gen, device=device).to(torch.bfloat16)
    outs = [torch.empty_like(q) for _ in caches]
    stream = torch.cuda.Stream(device)
    torch.cuda.synchronize()   # inputs were written on the default stream
    comm = torch.cuda.Stream(device)          # every collective, in one order on every rank
    lstreams = [torch.cuda.Stream(device) for _ in caches]
    gathered = [torch.cuda.Event() for _ in caches]   # layer i's output all-gather has read outs[i]

    def step(attend):
        main = torch.cuda.current_stream()
        for st in lstreams + [comm]:
            st.wait_stream(main)
        for cache, st in zip(caches, lstreams):
            with torch.cuda.stream(st):
                cache.reset_parameters()
        for c in range(n_chunks):
            for i, cache in enumerate(caches):
                k, kr, v = layers[i][c]
                if attend:
                    main.wait_stream(lstreams[i])          # the layer's previous commit
                    if world > 1 and c > 0:
                        main.wait_event(gathered[i])       # the previous chunk's gather of outs[i]
                    log_kv_chunk_attention(cache, q, k, v, D ** -0.5, 0.0, out=outs[i])
                    if world > 1:                          # the outputs' all-gather, beside the next layers
                        comm.wait_stream(main)
                        with torch.cuda.stream(comm):
                            gather_heads(outs[i], group)
                            gathered[i].record(comm)
                batch.begin(i, dict(k=k, v=v, k_raw=kr, span_ends=ends_host, span_ends_device=ends_dev), lstreams[i])
            with torch.cuda.stream(comm):
                batch.finish()
        for st in lstreams + [comm]:
            main.wait_stream(st)

    res = {}
    for mode in ("flush", "flush_attend"):
        with torch.no_grad(), torch.cuda.stream(stream):
            for _ in range(max(1, args.warmup)):
                step(mode == "flush_attend")
            torch.cuda.synchronize()
            # One CUDA graph per step (every collective captured in the same order on every
            # rank); released before the process group goes away.
            graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(graph, stream=stream):
                step(mode == "flush_attend")
            graph.replay()
            torch.cuda.synchronize()
            if world > 1:
                dist.barrier()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(stream)
            for _ in range(args.steps):
                graph.replay()
            e1.record(stream)
            torch.cuda.synchronize()
        del graph
        t = torch.tensor([e0.elapsed_time(e1)], device=device)
        if world > 1:
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
        res[mode] = t.item() * 1000.0 / args.steps
    assert all(c.read_status() == 0 for c in caches)
    return {"metric": "flush us per 2048-tok chunk/layer, one sequence KV-head-sharded", "unit": "us",
            "value": round(res["flush"] / flushes_per_step, 2), "higher_is_better": False,
            "n_gpus": world, "scaling": "strong", "groups_per_rank": hi - lo, "flushes_per_step": flushes_per_step,
            "exchange_bytes_per_chunk": batch.send.numel() * 4 * world,
            "flush_attend": {"metric": "sharded flush-and-attend prefill us per 2048-token chunk/layer (chunk "
                                       "attention of the rank's heads + output all-gather + add_recent)",
                             "unit": "us", "value": round(res["flush_attend"] / (cfg["layers"] * n_chunks), 2),
                             "heads_per_rank": H_local,
                             "gather_bytes_per_layer_chunk": q.numel() * q.element_size() * world},
            "timing": "CUDA-graph steps, layer flushes on per-layer streams, one span-part all-gather per chunk, "
                      "max over ranks",
            "config": {k: cfg[k] for k in ("workload", "layers", "groups", "head_dim", "clusters", "B", "recent",
                                           "granularity", "exact", "span_cap", "tokens")}}


# ---------------------------------------------------------------------------------------------- decode
DECODE = dict(workload="decode attention over a 32K compressed cache (BASELINE configs[3])", batch=64,
              heads=16, groups=8, head_dim=128, clusters=12, B=128, filled_levels=4, recent=2048, exact=256,
              span_cap=64, max_seq=32768, layers=28, distinct_layer_caches=2, geometric_p=0.1)


def prefill_decode_cache(torch, cfg, batch, device, cos, sin, seed):
    """A cache whose state is written directly: full merged levels, exact pool, full window.

    12 clusters x 4 full levels x B' slots per (sequence, KV group); slot counts
    w ~ Geometric(0.1) (support >= 1), each slot's mid anchor m uniform in
    [0, max_seq) with sum_wp = w * m (so the mid anchor is m), p_lo/p_hi = m;
    K/V ~ N(0, 1) in bf16; 256 valid exact rows; a 2048-token window.
    """
    from logkv_b200.cache import LogStructuredKVCache
    G, D = cfg["groups"], cfg["head_dim"]
    c = LogStructuredKVCache(
        (batch, G, cfg["max_seq"], D), (batch, G, cfg["max_seq"], D), B=cfg["B"], recent_size=cfg["recent"],
        device=device, dtype=torch.bfloat16, semantic_clusters=True, semantic_anchor_mode="mid",
        allocate_second_order=False, cluster_k_max=cfg["clusters"], semantic_flush_granularity=cfg["recent"],
        semantic_centroid_backend="parallel", semantic_replay_updates=True, alpha_exact_tokens=cfg["exact"],
        alpha_span_max_tokens=cfg["span_cap"], beta_novelty=True, beta_adaptive_merge=True, cos_cache=cos,
        sin_cache=sin, rope_n_elem=D)
    gen = torch.Generator(device=device)
    gen.manual_seed(seed)
    Lf, Bs = cfg["filled_levels"], c.B_prime
    lv = (slice(None), slice(None), slice(None), slice(0, Lf))
    c.level_k[lv].normal_(generator=gen)
    c.level_v[lv].normal_(generator=gen)
    u = torch.rand(c.level_w[lv].shape, generator=gen, device=device).clamp_min(1e-7)
    w = torch.floor(torch.log(u) / np.log(1.0 - cfg["geometric_p"])) + 1.0
    m = torch.randint(0, cfg["max_seq"], w.shape, generator=gen, device=device)
    c.level_w[lv] = w
    c.level_sum_wp[lv] = w.long() * m
    c.level_p_lo[lv] = m
    c.level_p_hi[lv] = m
    c.level_count[:, :, :, :Lf] = Bs
    P = cfg["exact"]
    c.alpha_k_raw.normal_(generator=gen)
    c.alpha_v.normal_(generator=gen)
    c.alpha_pos.copy_(torch.randint(0, cfg["max_seq"], c.alpha_pos.shape, generator=gen, device=device))
    c.alpha_valid.fill_(True)
    c._row_count.fill_(P)
    c._alpha_count_dev.fill_(P)
    R = cfg["recent"]
    c.recent_k[:, :, :R].normal_(generator=gen)
    c.recent_v[:, :, :R].normal_(generator=gen)
    c.recent_count = R
    c.token_count = cfg["max_seq"] // 2
    c._ladder_epoch += 1
    return c


def bench_decode(args, rank, world, local_rank):
    """Decode tokens/s: one new token per sequence attends over every layer's compressed cache."""
    import torch
    import torch.distributed as dist
    from logkv_b200.attention import log_kv_chunk_attention, refresh_prefix
    from logkv_b200.workload import rope_tables
    device = torch.device("cuda", local_rank)
    cfg = dict(DECODE, batch=args.decode_batch)
    batch = max(1, cfg["batch"] // world)
    H, G, D = cfg["heads"], cfg["groups"], cfg["head_dim"]
    cos_np, sin_np = rope_tables(cfg["max_seq"] + 1024, D, base=1e6)
    cos, sin = torch.from_numpy(cos_np).to(device), torch.from_numpy(sin_np).to(device)
    caches = [prefill_decode_cache(torch, cfg, batch, device, cos, sin, seed=100 * rank + i)
              for i in range(cfg["distinct_layer_caches"])]
    for c in caches:
        refresh_prefix(c)
    gen = torch.Generator(device=device)
    gen.manual_seed(7 + rank)
    q = torch.randn(batch, H, 1, D, generator=gen, device=device).to(torch.bfloat16)
    k = torch.randn(batch, G, 1, D, generator=gen, device=device).to(torch.bfloat16)
    v = torch.randn(batch, G, 1, D, generator=gen, device=device).to(torch.bfloat16)
    outs = [torch.empty(batch, H, 1, D, dtype=torch.bfloat16, device=device) for _ in range(cfg["layers"])]
    scale = D ** -0.5
    stream = torch.cuda.Stream(device)
    torch.cuda.synchronize()   # inputs were written on the default stream

    def step():
        for layer in range(cfg["layers"]):
            log_kv_chunk_attention(caches[layer % len(caches)], q, k, v, scale, 0.0, out=outs[layer])

    with torch.no_grad(), torch.cuda.stream(stream):
        for _ in range(max(3, args.warmup)):
            step()
        torch.cuda.synchronize()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=stream):
            step()
        for _ in range(2):
            graph.replay()
        torch.cuda.synchronize()
        n_steps = args.decode_steps
        if world > 1:
            dist.barrier()
        start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        with ClockSampler(local_rank) as clocks:
            start.record(stream)
            for _ in range(n_steps):
                graph.replay()
            stop.record(stream)
            torch.cuda.synchronize()
        ms = start.elapsed_time(stop)
        # Kernel-only view of one layer (for the roofline): the attention launch alone.
        one = torch.cuda.CUDAGraph()
        with torch.cuda.graph(one, stream=stream):
            log_kv_chunk_attention(caches[0], q, k, v, scale, 0.0, out=outs[0])
        one.replay()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        reps = 50
        e0.record(stream)
        for _ in range(reps):
            one.replay()
        e1.record(stream)
        torch.cuda.synchronize()
        layer_us = e0.elapsed_time(e1) * 1000.0 / reps
        # e2e: public API per layer, the step's q/k/v copied from pinned host memory, outputs read back.
        qh, kh, vh = (t.cpu().pin_memory() for t in (q, k, v))
        qd, kd_, vd = (torch.empty_like(t) for t in (q, k, v))
        host_out = torch.empty(cfg["layers"], batch, H, 1, D, dtype=torch.bfloat16).pin_memory()
        torch.cuda.synchronize()
        f0, f1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        f0.record(stream)
        for _ in range(n_steps):
            for layer in range(cfg["layers"]):
                for d_, h_ in ((qd, qh), (kd_, kh), (vd, vh)):
                    d_.copy_(h_, non_blocking=True)
                log_kv_chunk_attention(caches[layer % len(caches)], qd, kd_, vd, scale, 0.0, out=outs[layer])
                host_out[layer].copy_(outs[layer], non_blocking=True)
        f1.record(stream)
        torch.cuda.synchronize()
        e2e_ms = f0.elapsed_time(f1)
    del graph, one
    times = torch.tensor([ms, e2e_ms, layer_us], device=device)
    if world > 1:
        dist.all_reduce(times, op=dist.ReduceOp.MAX)
    ms, e2e_ms, layer_us = times.tolist()
    lengths = caches[0]._read.length.long()
    R = cfg["recent"]
    bytes_layer = int((lengths * (2 * D * 2 + 4)).sum().item()) + batch * G * (R * 2 * D * 2 + 2 * D * 2) \
        + 2 * batch * H * D * 2
    peak, peak_kind = measured_peaks()
    achieved = bytes_layer / (layer_us * 1e-6) / 1e9
    tokens = batch * world * n_steps
    step_bytes = (q.numel() + k.numel() + v.numel()) * 2
    return {"metric": "decode tok/s over a 32K compressed cache (28 layers)", "value": round(tokens / (ms / 1e3), 1),
            "unit": "tok/s", "n_gpus": world, "steps": n_steps, "batch": batch * world,
            "scaling": "strong", "us_per_layer_step": round(ms * 1000.0 / (n_steps * cfg["layers"]), 2),
            "slots_per_lane": int(lengths.float().mean().item()) + R + 1,
            "e2e": {"value": round(tokens / (e2e_ms / 1e3), 1), "unit": "tok/s",
                    "h2d_bytes_per_step": step_bytes * cfg["layers"],
                    "d2h_bytes_per_step": batch * H * D * 2 * cfg["layers"]},
            "roofline": {"bound": "hbm", "kernel": "slot_attn_mma_kernel", "achieved": round(achieved, 1), "peak": peak,
                         "peak_kind": peak_kind, "unit": "GB/s", "frac": round(achieved / peak, 4), "traffic": None,
                         "bytes_per_launch": bytes_layer, "launch_us": round(layer_us, 2)},
            "clocks": clocks.summary(), "gpu_launches": n_steps * cfg["layers"],
            "config": {k_: cfg[k_] for k_ in cfg}}


def bench_generate(args, rank, world, local_rank):
    """BASELINE configs[3] as the model runs it: 512 generated tokens per sequence, every layer's
    decode step through ``LogKVDecoder`` (the reference's pending-token pairing: attention over the
    cache and [pending, current], then add_recent of the pair; the first pair overflows the full
    2048-token window and flushes 2048 tokens, batch-wide).  Eager (every step's window length
    differs), device time, max over ranks.  The token inputs (q, k, k_raw, v) of every step are
    copied from pinned host memory and the last layer's output is read back every token, inside
    the timed region.  Layer caches are independent and identical in work, so when the 28 layers'
    caches do not all fit in memory the leg runs as many distinct caches as fit and reports the
    28-layer rate from the measured time per layer-token."""
    import torch
    import torch.distributed as dist
    from logkv_b200.attention import refresh_prefix
    from logkv_b200.decode import LogKVDecoder
    from logkv_b200.workload import rope_tables
    device = torch.device("cuda", local_rank)
    cfg = dict(DECODE, batch=args.decode_batch)
    batch = max(1, cfg["batch"] // world)
    H, G, D = cfg["heads"], cfg["groups"], cfg["head_dim"]
    n_tokens = args.generate_tokens
    cos_np, sin_np = rope_tables(cfg["max_seq"] + 1024, D, base=1e6)
    cos, sin = torch.from_numpy(cos_np).to(device), torch.from_numpy(sin_np).to(device)
    torch.cuda.synchronize()
    free0 = torch.cuda.mem_get_info(device)[0]
    first = prefill_decode_cache(torch, cfg, batch, device, cos, sin, seed=500 + rank)
    refresh_prefix(first)
    torch.cuda.synchronize()
    per_cache = max(1, free0 - torch.cuda.mem_get_info(device)[0])
    fit = int(0.8 * torch.cuda.mem_get_info(device)[0] // per_cache) + 1
    layers_real = max(1, min(cfg["layers"], fit))
    if world > 1:
        t = torch.tensor([layers_real], device=device)
        dist.all_reduce(t, op=dist.ReduceOp.MIN)
        layers_real = int(t.item())
    caches = [first] + [prefill_decode_cache(torch, cfg, batch, device, cos, sin, seed=500 + rank + 17 * i)
                        for i in range(1, layers_real)]
    for c in caches:
        refresh_prefix(c)
    scale = D ** -0.5
    decoders = [LogKVDecoder(c, scale) for c in caches]
    gen = torch.Generator(device="cpu").manual_seed(9 + rank)
    nsets = 8   # distinct token inputs, cycled
    host = [tuple(torch.randn(batch, n, 1, D, generator=gen).to(torch.bfloat16).pin_memory()
                  for n in (H, G, G, G)) for _ in range(nsets)]
    dev_in = [tuple(torch.empty_like(t, device=device) for t in host[0]) for _ in range(2)]
    ends_host = [[False] for _ in range(batch)]
    ends_dev = torch.zeros(batch, 1, dtype=torch.uint8, device=device)
    outs = [torch.empty(batch, H, 1, D, dtype=torch.bfloat16, device=device) for _ in caches]
    readback = torch.empty(batch, H, 1, D, dtype=torch.bfloat16).pin_memory()
    stream = torch.cuda.Stream(device)
    flushes0 = sum(c.read_counters()["flushes"] for c in caches)
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with torch.no_grad(), torch.cuda.stream(stream), ClockSampler(local_rank) as clocks:
        e0.record(stream)
        for t in range(n_tokens):
            buf = dev_in[t % 2]
            for d_, h_ in zip(buf, host[t % nsets]):
                d_.copy_(h_, non_blocking=True)
            q, k, kr, v = buf
            for dec, o in zip(decoders, outs):
                dec.step(q, k, v, k_raw=kr, span_ends=ends_host, span_ends_device=ends_dev, out=o)
            readback.copy_(outs[-1], non_blocking=True)
        e1.record(stream)
        torch.cuda.synchronize()
    ms = e0.elapsed_time(e1)
    t_ = torch.tensor([ms], device=device)
    if world > 1:
        dist.all_reduce(t_, op=dist.ReduceOp.MAX)
    ms = float(t_.item())
    flushes = sum(c.read_counters()["flushes"] for c in caches) - flushes0
    assert all(c.read_status() == 0 for c in caches)
    us_layer_token = ms * 1000.0 / (n_tokens * layers_real)
    tok_s = batch * world / (us_layer_token * cfg["layers"] * 1e-6)
    step_bytes = sum(t.numel() * t.element_size() for t in host[0])
    return {"metric": "decode tok/s over a 32K compressed cache (28 layers), generating with commits",
            "value": round(tok_s, 1), "unit": "tok/s", "n_gpus": world, "batch": batch * world,
            "tokens_per_sequence": n_tokens, "scaling": "strong", "us_per_layer_token": round(us_layer_token, 2),
            "layers_timed": layers_real, "flushes": flushes,
            "e2e": {"value": round(tok_s, 1), "unit": "tok/s", "h2d_bytes_per_step": step_bytes,
                    "d2h_bytes_per_step": readback.numel() * readback.element_size()},
            "timing": "eager steps (public LogKVDecoder API), host token inputs copied in and the last layer's "
                      "output read back every token, device time, max over ranks",
            "clocks": clocks.summary(),
            "config": {k_: cfg[k_] for k_ in cfg}}


def bench_prefill(args, rank, world, local_rank):
    """Chunk attention of one 2048-token chunk (16 q / 8 KV heads) over a pre-filled cache, per layer."""
    import torch
    import torch.distributed as dist
    from logkv_b200.attention import log_kv_chunk_attention, refresh_prefix
    from logkv_b200.workload import rope_tables
    device = torch.device("cuda", local_rank)
    cfg = dict(DECODE, batch=1)
    H, G, D, T = cfg["heads"], cfg["groups"], cfg["head_dim"], 2048
    cos_np, sin_np = rope_tables(cfg["max_seq"] + 1024, D, base=1e6)
    cos, sin = torch.from_numpy(cos_np).to(device), torch.from_numpy(sin_np).to(device)
    caches = [prefill_decode_cache(torch, cfg, 1, device, cos, sin, seed=500 + 100 * rank + i) for i in range(2)]
    for c in caches:
        refresh_prefix(c)
    gen = torch.Generator(device=device)
    gen.manual_seed(11 + rank)
    q = torch.randn(1, H, T, D, generator=gen, device=device).to(torch.bfloat16)
    k = torch.randn(1, G, T, D, generator=gen, device=device).to(torch.bfloat16)
    v = torch.randn(1, G, T, D, generator=gen, device=device).to(torch.bfloat16)
    out = torch.empty(1, H, T, D, dtype=torch.bfloat16, device=device)
    scale = D ** -0.5
    stream = torch.cuda.Stream(device)
    torch.cuda.synchronize()   # inputs were written on the default stream
    reps = max(4, args.decode_steps // 2)
    with torch.no_grad(), torch.cuda.stream(stream):
        for _ in range(3):
            log_kv_chunk_attention(caches[0], q, k, v, scale, 0.0, out=out)
        g1 = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g1, stream=stream):
            for layer in range(cfg["layers"]):
                log_kv_chunk_attention(caches[layer % 2], q, k, v, scale, 0.0, out=out)
        g1.replay()
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(reps):
            g1.replay()
        e1.record(stream)
        torch.cuda.synchronize()
        ms = e0.elapsed_time(e1)
    del g1
    t = torch.tensor([ms], device=device)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    us = t.item() * 1000.0 / (reps * cfg["layers"])
    Lp = int(caches[0]._read.length[0].float().mean().item())
    R = cfg["recent"]
    flops = 4.0 * D * H * (T * (Lp + R) + T * (T + 1) / 2)   # QK^T and PV over the visible slots
    peak, peak_kind = measured_peaks("bf16_tflops")
    tflops = flops / (us * 1e-6) / 1e12
    return {"metric": "chunk attention us per 2048-token chunk/layer", "value": round(us, 2), "unit": "us",
            "roofline": {"bound": "tensor", "kernel": "chunk_attn_tc_kernel", "achieved": round(tflops, 1),
                         "peak": peak, "peak_kind": peak_kind, "unit": "TFLOP/s", "frac": round(tflops / peak, 4),
                         "traffic": PREFILL_TRAFFIC, "flops_per_launch": flops},
            "config": {"heads": H, "groups": G, "head_dim": D, "chunk": T, "prefix_slots": Lp, "recent": R,
                       "layers": cfg["layers"], "distinct_layer_caches": 2}}


# ---------------------------------------------------------------------------------------------- CPU leg
def cpu_flush_sample(n_flushes: int = 3, seed: int = 7):
    """Time the oracle port on flushes of one layer of the same shape (single thread)."""
    from logkv_b200.workload import MixtureKeys, boundary_pattern
    from oracle.cache import OracleCache
    cfg = WORKLOAD
    rng = np.random.default_rng(seed)
    G, D, T = cfg["groups"], cfg["head_dim"], cfg["chunk"]
    mix = MixtureKeys(rng, G, D, cfg["clusters"])
    oc = OracleCache(batch=1, groups=G, max_seq=cfg["tokens"], dim=D, B=cfg["B"], recent=cfg["recent"],
                     clusters=cfg["clusters"], granularity=cfg["granularity"], exact=cfg["exact"],
                     span_cap=cfg["span_cap"], beta=cfg["beta"], dtype="bf16")
    times = []
    for c in range(n_flushes + 1):
        kr = mix.draw(1, T)
        v = rng.standard_normal((1, G, T, D)).astype(np.float32)
        pos = np.arange(c * T, (c + 1) * T)[None]
        ends = boundary_pattern(rng, 1, T, "mod23")
        t = time.perf_counter()
        oc.add_recent(kr, v, kr, pos, ends)
        if c:
            times.append(time.perf_counter() - t)
    return statistics.median(times) * 1e6, n_flushes


def _cpu_layer_worker(layer, steps, barrier):
    """One layer's oracle flushes in a worker process: `steps` flushes, one per step, each started
    after every worker has reached the step's barrier; returns the wall-clock (start, end) of every
    flush.  The next chunk is drawn before the barrier, and a stream that reaches the maximum
    sequence length restarts as a new stream (window refilled) outside the timed part."""
    from logkv_b200.workload import MixtureKeys, boundary_pattern
    from oracle.cache import OracleCache
    cfg = WORKLOAD
    rng = np.random.default_rng(1000 + layer)
    G, D, T = cfg["groups"], cfg["head_dim"], cfg["chunk"]
    mix = MixtureKeys(rng, G, D, cfg["clusters"])

    def chunk(c):
        kr = mix.draw(1, T)
        v = rng.standard_normal((1, G, T, D)).astype(np.float32)
        return kr, v, np.arange(c * T, (c + 1) * T)[None], boundary_pattern(rng, 1, T, "mod23")

    def new_stream():
        oc = OracleCache(batch=1, groups=G, max_seq=cfg["tokens"], dim=D, B=cfg["B"], recent=cfg["recent"],
                         clusters=cfg["clusters"], granularity=cfg["granularity"], exact=cfg["exact"],
                         span_cap=cfg["span_cap"], beta=cfg["beta"], dtype="bf16")
        kr, v, pos, ends = chunk(0)
        oc.add_recent(kr, v, kr, pos, ends)      # fills the window, no flush
        return oc, 1

    oc, c = new_stream()
    spans = []
    for _ in range(steps):
        if (c + 1) * T > cfg["tokens"]:
            oc, c = new_stream()
        kr, v, pos, ends = chunk(c)
        c += 1
        barrier.wait()
        t0 = time.time()
        oc.add_recent(kr, v, kr, pos, ends)      # one 2048-token flush
        spans.append((t0, time.time()))
    return spans


def cpu_flush_steps(warmup: int, steps: int):
    """The reference arm: the oracle port on every host core.  One worker process per layer
    (spawned, one BLAS thread each; the 28 layers' flushes are independent, so up to the core
    count run at once); a step is one flush in every worker, started together.  Returns
    (microseconds per flush, milliseconds per step, workers) over the `steps` timed steps that
    follow `warmup` untimed ones; a step's time runs from its first flush's start to its last
    flush's end."""
    import multiprocessing as mp
    workers = max(1, min(WORKLOAD["layers"], os.cpu_count() or 1))
    for var in ("OMP_NUM_THREADS", "OPENBLAS_NUM_THREADS", "MKL_NUM_THREADS"):
        os.environ[var] = "1"
    ctx = mp.get_context("spawn")
    with ctx.Manager() as manager:
        barrier = manager.Barrier(workers)
        with ctx.Pool(workers) as pool:
            spans = pool.starmap(_cpu_layer_worker, [(layer, warmup + steps, barrier) for layer in range(workers)])
    step_s = [max(sp[i][1] for sp in spans) - min(sp[i][0] for sp in spans) for i in range(warmup, warmup + steps)]
    total = sum(step_s)
    return total * 1e6 / (steps * workers), total * 1e3 / steps, workers


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=3)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--cpu-flushes", type=int, default=3, help="oracle flushes timed for cpu_baseline (0: skip)")
    ap.add_argument("--layers", type=int, default=WORKLOAD["layers"], help="layer caches (profiling runs only)")
    ap.add_argument("--decode-steps", type=int, default=32, help="timed decode steps (0: skip the decode leg)")
    ap.add_argument("--decode-batch", type=int, default=DECODE["batch"], help="decode sequences (profiling runs only)")
    ap.add_argument("--generate-tokens", type=int, default=512,
                    help="tokens generated per sequence in the decode-with-commits leg (0: skip it)")
    ap.add_argument("--streams", type=int, default=28, help="streams the layers' flushes are spread over")
    ap.add_argument("--flush-attend", type=int, default=1, help="run the flush-and-attend prefill leg (0: skip)")
    ap.add_argument("--unified", type=int, default=1, help="run the unified-route leg (0: skip)")
    ap.add_argument("--unified-streams", type=int, default=UNIFIED["streams_per_rank"],
                    help="streams per rank of the unified-route leg (profiling runs only)")
    ap.add_argument("--kv-layers", type=int, default=28,
                    help="layers of the KV-head-sharded leg (BASELINE configs[2]; 0 skips it)")
    args = ap.parse_args()
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    config = {k: WORKLOAD[k] for k in ("workload", "layers", "groups", "head_dim", "clusters", "B", "recent",
                                        "granularity", "exact", "span_cap", "tokens", "batch_per_rank")}
    config.update(layers=args.layers, parallelism=f"batch-sharded streams x{world}",
                  layer_streams=args.streams,
                  l2="inputs larger than L2 (5.6 GB per step at 28 layers)")
    if args.impl == "reference":
        if rank != 0:
            return
        us, ms_step, workers = cpu_flush_steps(args.warmup, args.steps)
        sample = (f"{args.steps} timed steps after {args.warmup} warm-up steps; a step = one 2048-token flush "
                  f"of each of {workers} layers, in parallel worker processes (oracle/ numpy port of the "
                  "reference's CPU path, one thread each); value = step time / flushes per step")
        line = dict(metric=METRIC, value=round(us, 1), unit="us", n_gpus=args.gpus, steps=args.steps,
                    warmup=args.warmup, ms_per_step=round(ms_step, 2), higher_is_better=False,
                    scaling="weak", vs_baseline=None, dtype="bf16", data="synthetic", config=config,
                    impl="reference", flushes_per_step=workers,
                    cpu_baseline={"value": round(us, 1), "unit": "us", "cores": workers, "kind": "port",
                                  "sample": sample},
                    e2e={"value": round(us, 1), "unit": "us", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0})
        print(json.dumps(line), flush=True)
        return
    import torch
    import torch.distributed as dist
    from logkv_b200 import build as _build
    if rank == 0 and not os.path.exists(os.path.join(ROOT, "logkv_b200", "liblogkv_b200.so")):
        _build.build()
    if world > 1:
        import datetime
        dist.init_process_group("nccl", device_id=torch.device("cuda", local_rank),
                                timeout=datetime.timedelta(seconds=180))
    res = bench_ours(args, rank, world, local_rank)
    inputs = res.pop("inputs")
    fa = bench_flush_attend(args, rank, world, local_rank, inputs) if args.flush_attend else None
    del inputs
    dec = bench_decode(args, rank, world, local_rank) if args.decode_steps > 0 else None
    if dec is not None and args.generate_tokens > 0:
        torch.cuda.empty_cache()
        dec["generate"] = bench_generate(args, rank, world, local_rank)
        torch.cuda.empty_cache()
    pre = bench_prefill(args, rank, world, local_rank) if args.decode_steps > 0 else None
    kvs = bench_kv_sharded(args, rank, world, local_rank) if args.kv_layers > 0 else None
    uni = bench_unified(args, rank, world, local_rank) if args.unified else None
    cpu = None
    if rank == 0 and world == 1 and args.cpu_flushes > 0:
        us, n = cpu_flush_sample(args.cpu_flushes)
        cpu = {"value": round(us, 1), "unit": "us", "cores": 1, "kind": "port",
               "sample": f"median of {n} flushes of one 0.6B-shaped layer (oracle/, numpy, 1 thread)"}
    if rank == 0:
        line = dict(metric=METRIC, value=round(res["value"], 2), unit="us", n_gpus=world, steps=args.steps,
                    warmup=args.warmup, ms_per_step=round(res["ms_per_step"], 3), higher_is_better=False,
                    scaling="weak", vs_baseline=None, dtype="bf16", data="synthetic", config=config,
                    e2e={"value": round(res["e2e_us"], 2), "unit": "us", "h2d_bytes_per_step": res["h2d"],
                         "d2h_bytes_per_step": 4 * args.layers * world},
                    roofline=res["roofline"], flush_roofline=res["flush_roofline"], cpu_baseline=cpu,
                    clocks=res["clocks"], gpu_launches=res["launches"], stages_us=res["stages"],
                    stages_us_median=res["stages_med"], stages_us_max=res["stages_max"],
                    flushes_per_step=res["flushes_per_step"],
                    rows_per_flush={k: round(v / res["flushes_per_step"], 1) for k, v in res["counters"].items()
                                    if k != "flushes"},
                    decode=dec, prefill=pre, flush_attend=fa, kv_sharded=kvs,
                    unified=uni, configs0_reference=configs0_reference_timing())
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
