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
