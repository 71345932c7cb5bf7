"""Token-by-token decoding over one layer's cache, as the reference's attention module runs it.

The reference commits decode tokens in pairs (litgpt/model.py:1219-1247, :1330-1352): a token
with no pending token attends over the frozen cache plus itself (causal) and becomes pending;
the next token's single query attends over the cache plus [pending, itself] (``causal_tail=0``)
and the pair is committed with ``add_recent``, which flushes ``semantic_flush_granularity``
tokens when the window overflows (the first pair after a full window does).  ``LogKVDecoder``
keeps the pending token in preallocated two-token buffers, so a step allocates nothing.
"""
from __future__ import annotations

import torch

from .attention import log_kv_chunk_attention


class LogKVDecoder:
    """Decode steps (one token per batch row) over ``cache``, with the reference's pending pairing."""

    def __init__(self, cache, scale: float):
        self.cache, self.scale = cache, float(scale)
        B, G = cache.batch_size, cache.n_groups
        dt, dev = cache.level_k.dtype, cache.level_k.device
        self._k = torch.zeros(B, G, 2, cache.k_dim, dtype=dt, device=dev)
        self._v = torch.zeros(B, G, 2, cache.v_dim, dtype=dt, device=dev)
        self._kr = torch.zeros(B, G, 2, cache.k_dim, dtype=dt, device=dev)
        self._pos = torch.zeros(B, 2, dtype=torch.int64, device=dev)
        self._ends = torch.zeros(B, 2, dtype=torch.uint8, device=dev)
        self._ends_host = None
        self._has_pos = False
        self.pending = False

    def reset(self) -> None:
        """Forget the pending token (the reference clears it with the cache, model.py:1180-1182)."""
        self.pending = False

    def step(self, q, k, v, *, k_raw, input_pos=None, span_ends=None, span_ends_device=None, out=None):
        """One token: q [B, H, 1, D], k / v / k_raw [B, G, 1, D]; returns the attention output
        [B, H, 1, D].  ``input_pos`` ([1] or [B, 1]) and the span-end flags (``span_ends`` host
        rows of one flag, or ``span_ends_device`` uint8 [B, 1]) follow add_recent's contract."""
        if q.size(2) != 1 or k.size(2) != 1:
            raise ValueError("decode steps take one token per batch row")
        slot = 1 if self.pending else 0
        self._k[:, :, slot:slot + 1].copy_(k)
        self._v[:, :, slot:slot + 1].copy_(v)
        self._kr[:, :, slot:slot + 1].copy_(k_raw)
        if input_pos is not None:
            pos = input_pos.reshape(1, 1) if input_pos.dim() == 1 else input_pos
            self._pos[:, slot:slot + 1].copy_(pos)
        if slot == 0:
            self._has_pos = input_pos is not None
            self._ends_host = [list(r) for r in span_ends] if span_ends is not None else None
        elif (input_pos is not None) != self._has_pos:
            raise ValueError("input_pos must be given for both tokens of a pair or for neither")
        if span_ends_device is not None:
            self._ends[:, slot:slot + 1].copy_(span_ends_device)
        if not self.pending:
            y = log_kv_chunk_attention(self.cache, q, k, v, self.scale, 0.0, reuse_prefix=True, out=out)
            self.pending = True
            return y
        y = log_kv_chunk_attention(self.cache, q, self._k, self._v, self.scale, 0.0, causal_tail=0,
                                   reuse_prefix=True, out=out)
        ends = [a + list(b) for a, b in zip(self._ends_host, span_ends)] \
            if (self._ends_host is not None and span_ends is not None) else None
        if ends is None:
            ends = [[False, False] for _ in range(self.cache.batch_size)]
        self.cache.add_recent(self._k, self._v, k_raw=self._kr, input_pos=self._pos if self._has_pos else None,
                              span_ends=ends, span_ends_device=self._ends if span_ends_device is not None else None)
        self.pending = False
        return y
