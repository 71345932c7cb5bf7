"""KV-head sharding of one long sequence over the GPUs of a node (one process per GPU).

Rank r of W holds the contiguous block of KV groups [r * G / W, (r + 1) * G / W) of every
layer's cache and the query heads that read them (GQA: head h reads group h // (H / G)).
Flush state, routing and the ladder are per (sequence, group) lane, so a rank flushes its
groups alone except for one exchange: the Alpha span score is a mean over all groups of
per-group parts (the Beta score the mean of the top two groups;
litgpt/alpha_log_kv.py:154-156, :173), so the ranks all-gather their parts before the
span choice (``gather_span_parts``) and every rank then makes the unsharded choice.
Attention of a chunk runs per rank on its heads; ``gather_heads`` all-gathers the
outputs into the full head order for the replicated projection that follows.

``BatchedFlush`` runs the flushes of many such caches (one model's layers, same geometry)
with ONE span-part exchange per chunk: every layer's score phase on its own stream, the
parts packed back to back, one all-gather, then every layer's commit on its stream.
"""
from __future__ import annotations

import torch
import torch.distributed as dist


def group_block(groups: int, rank: int, world: int) -> tuple[int, int]:
    """[start, stop) of the KV groups rank ``rank`` holds."""
    if groups % world:
        raise ValueError(f"{groups} KV groups do not split evenly over {world} ranks")
    per = groups // world
    return rank * per, (rank + 1) * per


def gather_span_parts(local: torch.Tensor, group=None, out: torch.Tensor | None = None) -> torch.Tensor:
    """All-gather each rank's flat span parts into ``[world * local.numel()]`` in rank order."""
    world = dist.get_world_size(group)
    if out is None:
        out = torch.empty(world * local.numel(), dtype=local.dtype, device=local.device)
    dist.all_gather_into_tensor(out, local.reshape(-1), group=group)
    return out


def gather_heads(out_local: torch.Tensor, group=None) -> torch.Tensor:
    """[B, H_local, T, D] per rank -> [B, world * H_local, T, D] in global head order."""
    world = dist.get_world_size(group)
    B, Hl = out_local.shape[:2]
    buf = torch.empty((world * B,) + tuple(out_local.shape[1:]), dtype=out_local.dtype, device=out_local.device)
    dist.all_gather_into_tensor(buf, out_local.contiguous(), group=group)
    buf = buf.view(world, B, *out_local.shape[1:])
    return buf.permute(1, 0, 2, 3, 4).reshape(B, world * Hl, *out_local.shape[2:])


class BatchedFlush:
    """The chunk commits of many KV-head-sharded caches with one span-part all-gather per chunk.

    ``begin(i, kwargs, stream)`` appends a chunk to cache i (``LogStructuredKVCache.
    add_recent_deferred``) on ``stream``, after the work queued so far on the caller's stream;
    when it flushes, the cache's span parts go to slot i of one send buffer.  ``finish(streams)``
    then exchanges every slot with one ``all_gather_into_tensor`` on the caller's stream
    ([world, caches, parts] after it) and runs every begun cache's commit on its stream, reading
    its parts of every rank at stride ``caches * parts``.  All caches of a batch share one
    geometry and chunk size, so they flush on the same chunks.  ``events[i]`` marks cache i's
    commit; ``wait_all`` makes the caller's stream wait for every commit.  Every collective is on
    the caller's stream, in the same order on every rank.  ``add_recent`` is begin for every
    cache followed by finish.
    """

    def __init__(self, caches, group=None):
        if not caches:
            raise ValueError("no caches")
        self.caches = list(caches)
        self.group = group
        self.world = dist.get_world_size(group) if (group is not None or dist.is_initialized()) else 1
        take = self.caches[0].semantic_flush_granularity
        self.count = self.caches[0]._local_parts(take).numel()
        for c in self.caches:
            if c._local_parts(take).numel() != self.count:
                raise ValueError("batched caches must share one geometry")
        dev = self.caches[0].level_k.device
        self.device = dev
        self.send = torch.zeros(len(self.caches) * self.count, dtype=torch.float32, device=dev)
        self.recv = torch.zeros(self.world * len(self.caches) * self.count, dtype=torch.float32, device=dev)
        self.events = [torch.cuda.Event() for _ in self.caches]
        self._recorded = []  # caches whose commit the last finish() recorded in self.events
        self._begun = {}     # cache index -> (stream, flushed)

    def begin(self, i: int, kwargs: dict, stream=None) -> None:
        main = torch.cuda.current_stream(self.device)
        st = stream or main
        if st is not main:
            st.wait_stream(main)
        with torch.cuda.stream(st):
            local = self.caches[i].add_recent_deferred(**kwargs)
            if local is not None:
                self.send[i * self.count:(i + 1) * self.count].copy_(local)
        self._begun[i] = (st, local is not None)

    def finish(self) -> bool:
        """Exchange and commit the begun caches' flushes; returns whether they flushed."""
        main = torch.cuda.current_stream(self.device)
        begun, self._begun = self._begun, {}
        for st, _ in begun.values():
            if st is not main:
                main.wait_stream(st)
        flushed = [i for i, (_, f) in begun.items() if f]
        self._recorded = flushed
        if not flushed:
            return False
        if len(flushed) != len(self.caches):
            raise RuntimeError("batched caches must flush on the same chunk")
        if self.world > 1:
            dist.all_gather_into_tensor(self.recv, self.send, group=self.group)
        stride = len(self.caches) * self.count
        for i in flushed:
            st = begun[i][0]
            if st is not main:
                st.wait_stream(main)
            with torch.cuda.stream(st):
                if self.world > 1:
                    self.caches[i].commit_deferred(self.recv[i * self.count:], self.world, stride)
                else:
                    self.caches[i].commit_deferred()
                self.events[i].record(st)
        return True

    def add_recent(self, chunks, streams=None) -> bool:
        """chunks[i]: keyword arguments of cache i's add_recent (k, v, k_raw, span_ends, ...).
        Returns whether the chunks flushed."""
        for i, kw in enumerate(chunks):
            self.begin(i, kw, streams[i % len(streams)] if streams else None)
        return self.finish()

    def wait_all(self) -> None:
        """The caller's stream waits for the commits of the last finish()."""
        main = torch.cuda.current_stream(self.device)
        for i in self._recorded:
            main.wait_event(self.events[i])
