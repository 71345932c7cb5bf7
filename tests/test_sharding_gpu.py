"""KV-head sharding on two GPUs: each rank flushes half the groups of the golden streams.

Two NCCL ranks (one process per GPU) each hold one of the streams' two KV groups.
After every ``add_recent`` each rank's buffers must equal the reference fixture's
slice of its group bit for bit (the span choice is made from all ranks' gathered
parts), the shared exact-pool positions and host mirrors must match, and the
chunk attention of the rank's heads, all-gathered, must match the reference's
attention within the bf16/fp32 tolerance.  Skipped with fewer than two GPUs.
"""
from __future__ import annotations

import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu

FIELDS = ["level_count", "alive", "p_hi_c", "n_total", "level0_phase", "level_p_lo", "level_p_hi", "level_sum_wp",
          "level_order", "pad_mask", "level_w", "level_k", "level_v", "alpha_k_raw", "alpha_v", "recent_k",
          "recent_k_raw", "recent_v", "centroid", "n_eff"]
SHARED = ["alpha_pos", "alpha_valid", "recent_pos"]
TOL = {"bf16": 2e-2, "fp32": 1e-4}


def free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def worker(rank: int, world: int, port: int, name: str, out: dict) -> None:
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=torch.device("cuda", rank))
    try:
        from fixtures import as_values, config, load, make_stream
        from logkv_b200 import log_kv_chunk_attention
        from logkv_b200.cache import LogStructuredKVCache
        from logkv_b200.sharding import gather_heads, group_block
        cfg = config(name)
        stream = make_stream(cfg)
        ref_steps = load(name)
        dt = torch.float32 if cfg["dtype"] == "fp32" else torch.bfloat16
        g0, g1 = group_block(cfg["groups"], rank, world)
        rf = 2
        cos, sin = torch.from_numpy(stream["cos"]), torch.from_numpy(stream["sin"])
        if cfg.get("rope_dtype", "fp32") == "bf16":
            cos, sin = cos.to(torch.bfloat16), sin.to(torch.bfloat16)
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
        errors = []
        for step, (chunk, ref) in enumerate(zip(stream["chunks"], ref_steps)):
            sl = slice(g0, g1)
            k = torch.from_numpy(chunk["k"][:, sl]).to(dev, dt)
            kr = torch.from_numpy(chunk["k_raw"][:, sl]).to(dev, dt)
            v = torch.from_numpy(chunk["v"][:, sl]).to(dev, dt)
            if chunk["attend"]:
                q = torch.from_numpy(chunk["q"][:, g0 * rf:g1 * rf]).to(dev, dt)
                with torch.no_grad():
                    att = gather_heads(log_kv_chunk_attention(cache, q, k, v, cfg["dim"] ** -0.5, 0.0))
                err = np.abs(att.float().cpu().numpy() - ref["attention"]).max()
                if err > TOL[cfg["dtype"]]:
                    errors.append(f"step {step} attention {err}")
            pos = torch.from_numpy(chunk["pos"]).to(dev) if chunk.get("pos") is not None else None
            cache.add_recent(k, v, k_raw=kr, input_pos=pos, span_ends=chunk["span_ends"].tolist())
            for field in FIELDS + SHARED:
                want = as_values(ref[field], field)
                if field not in SHARED:
                    want = want[:, sl]
                got = getattr(cache, field).detach().cpu()
                got = (got.float() if got.dtype == torch.bfloat16 else got).numpy()
                if not np.array_equal(got.astype(want.dtype), want):
                    errors.append(f"step {step} {field}")
            if [cache.alpha_count, cache.recent_count, cache.token_count] != ref["scalars"].tolist()[:3]:
                errors.append(f"step {step} scalars")
        out[rank] = errors
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason="needs two GPUs")
@pytest.mark.parametrize("name", ["fp32_beta", "fp32_alpha", "bf16_beta"])
def test_kv_head_sharded_flush_matches_reference(name):
    ctx = mp.get_context("spawn")
    out = ctx.Manager().dict()
    mp.spawn(worker, args=(2, free_port(), name, out), nprocs=2, join=True)
    assert dict(out) == {0: [], 1: []}
