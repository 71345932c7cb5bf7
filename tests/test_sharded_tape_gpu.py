"""Update tape of a KV-head-sharded cache: record, reset, replay without an exchange.

Each NCCL rank (two when two GPUs are visible, else one rank, which still takes the sharded
path: scores, span-part all-gather, commit) holds its block of the golden stream's KV groups.
Every flush of the stream is recorded under ``_semantic_update_context`` with
``record_op_log=True`` (``logkv_flush_commit_record``: the commit half of the sharded flush
writes the rank's record); the recorded run must equal the reference fixture's slice of the
rank's groups.  After a reset the stream is replayed from the records: no flush is routed and
no span parts are exchanged (the record holds the ranks' common span choice), and every buffer
must equal the recorded run's after every step, bit for bit.
"""
from __future__ import annotations

import os
from unittest.mock import patch

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from test_sharding_gpu import FIELDS, SHARED, free_port

pytestmark = pytest.mark.gpu


def worker(rank: int, world: int, port: int, name: str, out: dict) -> None:
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=torch.device("cuda", rank))
    try:
        from fixtures import as_values, config, load, make_stream
        from logkv_b200 import _SemanticReplayUpdates
        from logkv_b200.cache import LogStructuredKVCache
        from logkv_b200.sharding import group_block
        cfg = config(name)
        stream = make_stream(cfg)
        ref_steps = load(name)
        dt = torch.float32 if cfg["dtype"] == "fp32" else torch.bfloat16
        g0, g1 = group_block(cfg["groups"], rank, world)
        cos, sin = torch.from_numpy(stream["cos"]), torch.from_numpy(stream["sin"])
        shape = (cfg["batch"], g1 - g0, cfg["max_seq"], cfg["dim"])
        cache = LogStructuredKVCache(
            shape, shape, B=cfg["slots"], recent_size=cfg["recent"], device=f"cuda:{rank}", dtype=dt,
            semantic_clusters=True, semantic_anchor_mode="mid", allocate_second_order=False,
            cluster_k_max=cfg["clusters"], semantic_flush_granularity=cfg["granularity"],
            semantic_centroid_backend="sequential", semantic_replay_updates=True,
            alpha_exact_tokens=cfg["exact"], alpha_span_max_tokens=cfg["span_cap"], beta_novelty=cfg["beta"],
            beta_adaptive_merge=cfg["beta"], semantic_s_h=cfg.get("s_h"), cos_cache=cos, sin_cache=sin,
            rope_n_elem=cfg["dim"], kv_shard_group=dist.group.WORLD)
        dev = torch.device("cuda", rank)
        sl = slice(g0, g1)

        def push(chunk, **kw):
            k = torch.from_numpy(chunk["k"][:, sl]).to(dev, dt)
            kr = torch.from_numpy(chunk["k_raw"][:, sl]).to(dev, dt)
            v = torch.from_numpy(chunk["v"][:, sl]).to(dev, dt)
            pos = torch.from_numpy(chunk["pos"]).to(dev) if chunk.get("pos") is not None else None
            cache.add_recent(k, v, k_raw=kr, input_pos=pos, span_ends=chunk["span_ends"].tolist(), **kw)

        def snapshot():
            return {n: x.clone() for n, x in cache.named_buffers()}

        errors, recorded = [], []
        tape = _SemanticReplayUpdates()
        with torch.no_grad(), cache._semantic_update_context(tape):
            for step, (chunk, ref) in enumerate(zip(stream["chunks"], ref_steps)):
                push(chunk, record_op_log=True)
                recorded.append(snapshot())
                for field in FIELDS + SHARED:
                    want = as_values(ref[field], field)
                    if field not in SHARED:
                        want = want[:, sl]
                    got = getattr(cache, field).detach().cpu()
                    got = (got.float() if got.dtype == torch.bfloat16 else got).numpy()
                    if not np.array_equal(got.astype(want.dtype), want):
                        errors.append(f"record step {step} {field}")
        if not tape.tensors:
            errors.append("nothing recorded")
        cache.reset_parameters()
        no_route = patch.object(cache, "flush_device", side_effect=AssertionError("rerouted"))
        no_exchange = patch.object(cache, "_gather_parts", side_effect=AssertionError("exchanged"))
        with no_route, no_exchange:
            for step, (chunk, want) in enumerate(zip(stream["chunks"], recorded)):
                with torch.no_grad(), cache._semantic_update_context(tape, replay=True):
                    push(chunk)
                if cache.read_status() != 0:
                    errors.append(f"replay step {step} status")
                for n, x in cache.named_buffers():
                    if not torch.equal(x, want[n]):
                        errors.append(f"replay step {step} {n}")
        out[rank] = errors
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(not torch.cuda.is_available(), reason="needs a GPU")
@pytest.mark.parametrize("name", ["fp32_beta", "bf16_beta"])
def test_sharded_update_tape_replays_without_exchange(name):
    world = min(2, torch.cuda.device_count())
    ctx = mp.get_context("spawn")
    out = ctx.Manager().dict()
    mp.spawn(worker, args=(world, free_port(), name, out), nprocs=world, join=True)
    assert dict(out) == {r: [] for r in range(world)}
