"""KV-head sharding host logic on CPU: two gloo ranks (no GPU).

The layout contract between ``sharding.gather_span_parts`` and the greedy kernel
(include/logkv_b200.h, logkv_flush_commit): rank r's parts [B, NC, G_local, 2] land
at [r] of a [ranks, B, NC, G_local, 2] buffer, so global group r * G_local + gl is read
at ((r * B + b) * NC + c) * G_local + gl.  Heads gather back into global order.
"""
from __future__ import annotations

import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp


def free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def worker(rank: int, world: int, port: int, out: dict) -> None:
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from logkv_b200.sharding import gather_heads, gather_span_parts, group_block
        B, NC, G, D, T, rf = 2, 7, 8, 16, 3, 2
        g0, g1 = group_block(G, rank, world)
        gl = g1 - g0
        gen = torch.Generator().manual_seed(5)
        full = torch.randn(B, NC, G, 2, generator=gen)
        gathered = gather_span_parts(full[:, :, g0:g1].contiguous(), None).view(world, B, NC, gl, 2)
        flat = gathered.reshape(-1)
        ok = True
        for grp in range(G):
            r, j = divmod(grp, gl)
            for b in range(B):
                for c in range(NC):
                    base = (((r * B + b) * NC + c) * gl + j) * 2
                    ok &= bool(torch.equal(flat[base:base + 2], full[b, c, grp]))
        heads = torch.randn(B, G * rf, T, D, generator=gen)
        local = heads[:, g0 * rf:g1 * rf].contiguous()
        ok &= bool(torch.equal(gather_heads(local, None), heads))
        out[rank] = ok
    finally:
        dist.destroy_process_group()


def test_group_block_splits_evenly():
    from logkv_b200.sharding import group_block
    assert [group_block(8, r, 4) for r in range(4)] == [(0, 2), (2, 4), (4, 6), (6, 8)]
    with pytest.raises(ValueError):
        group_block(8, 0, 3)


def test_two_rank_gathers_follow_global_group_order():
    ctx = mp.get_context("spawn")
    manager = ctx.Manager()
    out = manager.dict()
    mp.spawn(worker, args=(2, free_port(), out), nprocs=2, join=True)
    assert dict(out) == {0: True, 1: True}


def batched_worker(rank: int, world: int, port: int, out: dict) -> None:
    """Many layers' parts packed back to back, one all-gather: layer i of rank r is read at
    r * (layers * parts) + i * parts, the strided layout logkv_flush_commit_strided reads."""
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        layers, parts = 5, 11
        gen = torch.Generator().manual_seed(7)
        every = torch.randn(world, layers, parts, generator=gen)   # [rank, layer, parts]
        send = every[rank].reshape(-1).contiguous()
        recv = torch.empty(world * layers * parts)
        dist.all_gather_into_tensor(recv, send)
        stride = layers * parts
        ok = True
        for i in range(layers):
            base = recv[i * parts:]
            for r in range(world):
                ok &= bool(torch.equal(base[r * stride:r * stride + parts], every[r, i]))
        out[rank] = ok
    finally:
        dist.destroy_process_group()


def test_batched_gather_layout_matches_strided_commit():
    ctx = mp.get_context("spawn")
    manager = ctx.Manager()
    out = manager.dict()
    mp.spawn(batched_worker, args=(2, free_port(), out), nprocs=2, join=True)
    assert dict(out) == {0: True, 1: True}
