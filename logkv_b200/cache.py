"""B200 LogStructuredKVCache for the in-scope SemanticLogKV configuration.

Drop-in for the reference's ``LogStructuredKVCache`` (litgpt/log_kv_cache.py:640)
when it runs the default flush-and-attend route: semantic clusters with
K > 1, mid anchors, attach routing, the Alpha exact-span pool with or without
Beta, first-order entries.  The constructor takes the reference's keyword
arguments, registers the same buffers (same names, shapes, dtypes and
layout, so ``named_buffers()`` compares one-to-one), and ``add_recent`` keeps
the reference's window/flush contract (:5668-5718, :5609-5666).  Every flush
runs on the device through ``logkv_flush`` of the C-ABI library without a
host synchronization; the reference's host mirrors (``_semantic_counts``,
``_alpha_spans`` ...) are materialized from the device on attribute access.
"""
from __future__ import annotations

import contextlib
import ctypes
import math
import os

import numpy as np
import torch
import torch.nn as nn

from . import _lib

UNSUPPORTED = "logkv_b200 implements the attach or unified route + Alpha (+ Beta) mid-anchor flush path only"


def ladder_geometry(max_seq_length: int, k_dim: int, v_dim: int, n_groups: int, B: int, clusters: int,
                    exact: int, element_size: int) -> tuple[int, int]:
    """(B', L): slots per level after paying for the exact pool, and the level count.

    Same byte budget as the reference constructor (log_kv_cache.py:855-899):
    the largest B' < B whose ladder plus the exact pool fits in the ladder of B.
    """
    levels = max(2, math.ceil(math.log2(max_seq_length / max(clusters * B, 1) + 1.0)) + 2)
    if not exact:
        return B, levels
    packed_dim = ((max(k_dim + 1, v_dim) + 7) // 8) * 8
    entry = (k_dim + v_dim + 2 * packed_dim) * element_size + 41
    exact_bytes = exact * (n_groups * (k_dim + v_dim + 2 * packed_dim) * element_size + 9)
    baseline = n_groups * clusters * levels * (B * entry + 2)
    for cand in range(B - 1, 1, -1):
        lv = max(2, math.ceil(math.log2(max_seq_length / (clusters * cand) + 1.0)) + 2)
        if n_groups * clusters * lv * (cand * entry + 2) + exact_bytes <= baseline:
            return cand, lv
    raise ValueError("compressed ladder budget is too small for alpha_exact_tokens; increase B or reduce exact capacity")


class _SemanticReplayUpdates:
    """Update tape of one training invocation (the reference's _SemanticReplayUpdates,
    litgpt/log_kv_cache.py:111-137): one device record per flush, written by
    ``logkv_flush_record`` and applied by ``logkv_flush_replay``.

    ``flushes`` maps a flush key (the cache's flush index since its last reset, the flushed
    token count and the window fill) to (signature, tensor index, ready event); ``tensors``
    holds the device records.
    """

    def __init__(self, flushes=None, tensors=None):
        self.flushes = {} if flushes is None else flushes
        self.tensors = [] if tensors is None else tensors

    def wait(self, device):
        """Make the current stream wait until every record has been written (no host sync)."""
        if torch.device(device).type == "cuda":
            stream = torch.cuda.current_stream(device)
            for record in self.flushes.values():
                if record[-1] is not None:
                    stream.wait_event(record[-1])

    def save(self, tensor, owned=False):
        if tensor is None:
            return None
        index = len(self.tensors)
        self.tensors.append(tensor.detach() if owned else tensor.detach().clone())
        return index


class LogStructuredKVCache(nn.Module):
    # Route decisions beside the attention on a side stream (the reference's LOGKV_ROUTE_OVERLAP,
    # log_kv_cache.py:3814-3849): the flush's decision kernels wait only for the end of the
    # previous flush of this cache, not for the work queued on the caller's stream since then.
    _route_overlap = os.environ.get("LOGKV_ROUTE_OVERLAP", "0") == "1"
    _ROUTE_STREAMS: dict = {}

    def __init__(self, k_shape, v_shape, B: int = 512, recent_size: int = 0, device=None, dtype=None,
                 importance_pooling: bool = False, importance_pooling_lambda: float = 1.0,
                 importance_pooling_temperature: float = 1.0, semantic_clusters: bool = False,
                 cluster_k_max: int = 1, cluster_lambda_rel: float = 1.0, seg_eta: float = 1.0,
                 seg_g0: float = 2048.0, seg_gap_max=None, seg_block_level: int = 0, seg_forget: float = 0.5,
                 semantic_s_h=None, semantic_flush_granularity: int = 2, semantic_cluster_chunk_size: int = 0,
                 semantic_capacity_beta: float = 0.0, semantic_capacity_hard_cap_mult: float = 0.0,
                 semantic_legacy_route: bool = False, semantic_unified_route: bool = False,
                 semantic_merge_passes: int = 1, semantic_anchor_mode: str = "multi",
                 semantic_pack_backend: str = "auto", semantic_centroid_backend: str = "sequential",
                 semantic_replay_updates: bool = False, cos_cache=None, sin_cache=None, rope_n_elem=None,
                 allocate_second_order: bool = True, alpha_exact_tokens: int = 0, alpha_span_max_tokens: int = 64,
                 beta_novelty: bool = False, beta_adaptive_merge: bool = False, *, kv_shard_group=None) -> None:
        """The reference's constructor (litgpt/log_kv_cache.py:681-720): same keywords, order and
        defaults, so an unknown or misspelt keyword raises TypeError.  ``kv_shard_group`` (keyword
        only, no reference counterpart) makes this cache one rank's block of groups of a
        KV-head-sharded sequence."""
        super().__init__()
        batch, groups, max_seq, k_dim = k_shape
        v_dim = v_shape[3]
        device = torch.device(device) if device is not None else torch.device("cuda")
        dtype = dtype or torch.float32
        if dtype not in _lib.DTYPE_CODES:
            raise ValueError(f"storage dtype {dtype} is not supported (float32 or bfloat16)")
        if not semantic_clusters or semantic_anchor_mode != "mid" or allocate_second_order:
            raise NotImplementedError(UNSUPPORTED)
        if int(semantic_merge_passes) < 1:
            raise ValueError("semantic_merge_passes must be >= 1")
        if semantic_unified_route and (semantic_legacy_route or semantic_cluster_chunk_size):
            raise ValueError("unified routing requires semantic clusters and excludes legacy/chunk-tree routing")
        if semantic_unified_route and semantic_capacity_beta != 0.0:
            raise ValueError("unified routing uses Ward costs; semantic_capacity_beta must be 0")
        if semantic_legacy_route or semantic_cluster_chunk_size:
            raise NotImplementedError(UNSUPPORTED + " (attach or unified route)")
        if semantic_capacity_hard_cap_mult or semantic_capacity_beta or importance_pooling:
            raise NotImplementedError(UNSUPPORTED + " (no capacity terms)")
        if (seg_gap_max is not None and math.isfinite(seg_gap_max)) or seg_block_level:
            raise ValueError("AlphaLogKV requires disabled segment gaps/padding for delayed archival")
        if beta_novelty != beta_adaptive_merge:
            raise NotImplementedError(UNSUPPORTED + " (Beta novelty and 4->2 merge together)")
        if not alpha_exact_tokens:
            raise NotImplementedError(UNSUPPORTED + " (alpha_exact_tokens > 0)")
        if cluster_k_max <= 1 or cluster_k_max > 32:
            raise ValueError("cluster_k_max must be in [2, 32]")
        if k_dim != v_dim:
            raise NotImplementedError(UNSUPPORTED + " (k_dim == v_dim)")
        if not 1 <= alpha_span_max_tokens <= alpha_exact_tokens:
            raise ValueError("alpha_span_max_tokens must be in [1, alpha_exact_tokens]")
        if cos_cache is None or sin_cache is None or rope_n_elem is None:
            raise ValueError("semantic LogKV requires cos_cache, sin_cache, and rope_n_elem")
        if semantic_centroid_backend not in ("sequential", "parallel"):
            raise ValueError("semantic_centroid_backend must be sequential or parallel")
        self.recent_size = recent_size if recent_size > 0 else 2
        if not 1 <= semantic_flush_granularity <= self.recent_size:
            raise ValueError("semantic_flush_granularity must be in [1, recent_size]")
        if not (math.isfinite(cluster_lambda_rel) and cluster_lambda_rel > 0):
            raise ValueError("cluster_lambda_rel must be finite and > 0")
        if not (math.isfinite(seg_g0) and seg_g0 > 0):
            raise ValueError("seg_g0 must be finite and > 0")
        self.batch_size, self.n_groups, self.max_seq_length = batch, groups, max_seq
        self.k_dim, self.v_dim, self.B = k_dim, v_dim, B
        self.semantic_clusters = True
        self.semantic_anchor_mode = "mid"
        self.semantic_pack_backend = semantic_pack_backend
        self.semantic_centroid_backend = semantic_centroid_backend
        self.semantic_replay_updates = bool(semantic_replay_updates)
        self.semantic_unified_route = bool(semantic_unified_route)
        self.semantic_merge_passes = int(semantic_merge_passes)
        self.K_max = int(cluster_k_max)
        self.cluster_lambda_rel, self.seg_eta, self.seg_g0 = float(cluster_lambda_rel), float(seg_eta), float(seg_g0)
        self.seg_forget = float(seg_forget)
        self.semantic_flush_granularity = int(semantic_flush_granularity)
        self.alpha_exact_tokens, self.alpha_span_max_tokens = int(alpha_exact_tokens), int(alpha_span_max_tokens)
        self.beta_novelty, self.beta_adaptive_merge = bool(beta_novelty), bool(beta_adaptive_merge)
        self.rope_n_elem = int(rope_n_elem)
        self.allocate_second_order = False
        esize = torch.empty((), dtype=dtype).element_size()
        # A KV-head shard sizes its ladder like the whole cache (the exact pool's budget term
        # is not proportional to the group count).
        geo_groups = groups
        if kv_shard_group is not None:
            if semantic_unified_route:
                raise NotImplementedError(UNSUPPORTED + " (KV-head sharding of the attach route only)")
            import torch.distributed as dist
            geo_groups = groups * dist.get_world_size(kv_shard_group)
        self.B_prime, self.L_alloc = ladder_geometry(max_seq, k_dim, v_dim, geo_groups, B, self.K_max,
                                                     self.alpha_exact_tokens, esize)
        self.max_levels = self.L_alloc
        self.B = self.B_prime
        self.recent_capacity = 2 * self.recent_size
        self.slot_k_dim = int(cos_cache.size(1)) + k_dim - self.rope_n_elem
        self.token_count = 0
        self.recent_count = 0
        P, R, K, L, Bs = self.alpha_exact_tokens, self.recent_capacity, self.K_max, self.L_alloc, self.B_prime
        z = dict(device=device)
        reg = lambda name, t: self.register_buffer(name, t, persistent=False)  # noqa: E731
        reg("cos_cache", cos_cache.to(device=device))
        reg("sin_cache", sin_cache.to(device=device))
        reg("recent_k", torch.zeros(batch, groups, R, self.slot_k_dim, dtype=dtype, **z))
        reg("recent_v", torch.zeros(batch, groups, R, v_dim, dtype=dtype, **z))
        reg("recent_k_raw", torch.zeros(batch, groups, R, k_dim, dtype=dtype, **z))
        reg("recent_pos", torch.zeros(batch, R, dtype=torch.int64, **z))
        reg("alpha_k_raw", torch.zeros(batch, groups, P, k_dim, dtype=dtype, **z))
        reg("alpha_v", torch.zeros(batch, groups, P, v_dim, dtype=dtype, **z))
        reg("alpha_pos", torch.zeros(batch, P, dtype=torch.int64, **z))
        reg("alpha_valid", torch.zeros(batch, P, dtype=torch.bool, **z))
        shape = (batch, groups, K, L, Bs)
        reg("level_k", torch.zeros(*shape, k_dim, dtype=dtype, **z))
        reg("level_v", torch.zeros(*shape, v_dim, dtype=dtype, **z))
        reg("level_w", torch.zeros(*shape, dtype=torch.float32, **z))
        reg("level_imp", torch.zeros(*shape, dtype=torch.float32, **z))
        for name in ("level_sigma_u", "level_sigma2", "level_gamma_a", "level_gamma_b", "level_gamma"):
            reg(name, None)
        reg("level_count", torch.zeros(batch, groups, K, L, dtype=torch.int16, **z))
        reg("pad_mask", torch.zeros(*shape, dtype=torch.bool, **z))
        i64max = torch.iinfo(torch.int64).max
        reg("level_p_lo", torch.full(shape, i64max, dtype=torch.int64, **z))
        reg("level_p_hi", torch.full(shape, -1, dtype=torch.int64, **z))
        reg("level_sum_wp", torch.zeros(shape, dtype=torch.int64, **z))
        reg("level_order", torch.zeros(shape, dtype=torch.int64, **z))
        reg("centroid", torch.zeros(batch, groups, K, k_dim, dtype=torch.float32, **z))
        reg("n_eff", torch.zeros(batch, groups, K, dtype=torch.float32, **z))
        reg("n_total", torch.zeros(batch, groups, K, dtype=torch.int32, **z))
        reg("p_hi_c", torch.full((batch, groups, K), -1, dtype=torch.int64, **z))
        reg("current_segment", torch.zeros(batch, groups, K, dtype=torch.int32, **z))
        reg("level0_phase", torch.zeros(batch, groups, K, dtype=torch.int32, **z))
        reg("alive", torch.zeros(batch, groups, K, dtype=torch.bool, **z))
        reg("ward_cost", torch.full((batch, groups, K, K), float("inf"), dtype=torch.float32, **z))
        if semantic_s_h is None:
            s_h = torch.ones(batch, groups, dtype=torch.float32, **z)
        elif isinstance(semantic_s_h, torch.Tensor):
            s_h = semantic_s_h.to(device=device, dtype=torch.float32)
            if s_h.shape == (groups,):
                s_h = s_h.unsqueeze(0).expand(batch, -1).contiguous()
            elif s_h.shape != (batch, groups):
                raise ValueError(f"semantic_s_h must have shape ({groups},) or ({batch},{groups})")
        else:
            s_h = torch.full((batch, groups), float(semantic_s_h), dtype=torch.float32, **z)
        if not bool(torch.isfinite(s_h).all()) or not bool((s_h > 0).all()):
            raise ValueError("semantic_s_h must be finite and > 0")
        reg("s_h", s_h)
        # Device form of the reference's host-side pool lists (not registered buffers).
        self._recent_ends = torch.zeros(batch, R, dtype=torch.uint8, **z)
        self._ends_stage = torch.zeros(batch * R, dtype=torch.uint8, **z)   # host span-end lists, staged
        self._span_len = torch.zeros(batch, P, dtype=torch.int32, **z)
        self._span_closed = torch.zeros(batch, P, dtype=torch.uint8, **z)
        self._span_count = torch.zeros(batch, dtype=torch.int32, **z)
        self._row_count = torch.zeros(batch, dtype=torch.int32, **z)
        self._alpha_count_dev = torch.zeros(1, dtype=torch.int32, **z)
        self.op_log = None
        self.op_log_len = None
        self._layout = _lib.Layout(batch, groups, k_dim, K, L, Bs, R, P, self.alpha_span_max_tokens,
                                   int(self.beta_adaptive_merge), _lib.DTYPE_CODES[dtype], self.seg_eta,
                                   self.seg_g0, self.cluster_lambda_rel,
                                   _lib.ROUTE_UNIFIED if self.semantic_unified_route else _lib.ROUTE_ATTACH,
                                   self.semantic_merge_passes)
        nbytes = _lib.lib().logkv_flush_workspace_bytes(ctypes.byref(self._layout), self.semantic_flush_granularity)
        if not nbytes:
            raise ValueError("cache geometry is outside the supported range of the flush kernels")
        self._workspace = torch.zeros(nbytes, dtype=torch.uint8, device=device)
        self._state = None
        # KV-head sharding: this cache holds one rank's block of groups of a longer group axis
        # (logkv_b200.sharding); flushes exchange span parts over `kv_shard_group`.
        self.kv_shard_group = kv_shard_group
        self._span_gather = None
        self._ladder_epoch = 0       # bumped whenever a flush or reset rewrites the ladder / exact pool
        self._flush_cursor = 0       # flushes since the last reset (orders update-tape records)
        self._active_updates = None  # update tape being recorded or replayed
        self._replaying_updates = False
        self._update_actions = None
        self.profile_events = None   # set to a list of LOGKV_FLUSH_STAGES+1 torch.cuda.Event to time stages
        self._route_ready = None     # end of the last flush (route overlap), with the window rows it had
        self._route_ready_rows = 0
        self._route_ready_capture = 0
        self._route_done = None
        self._deferred_take = None   # flush started by add_recent_deferred, committed by commit_deferred

    # ------------------------------------------------------------------ C-ABI state
    def _apply(self, fn, *args, **kwargs):
        self._state = None           # buffers move: the pointer table is rebuilt on next use
        return super()._apply(fn, *args, **kwargs)

    def _state_struct(self) -> _lib.State:
        """Device pointers of every state buffer (built once; rebuilt when the buffers move)."""
        st = self._state
        if st is not None and st.level_k == self.level_k.data_ptr() and st.recent_k == self.recent_k.data_ptr():
            return st
        views = dict(level_k=self.level_k, level_v=self.level_v, level_w=self.level_w,
                     level_p_lo=self.level_p_lo, level_p_hi=self.level_p_hi, level_sum_wp=self.level_sum_wp,
                     level_order=self.level_order, pad_mask=self.pad_mask, level_count=self.level_count,
                     centroid=self.centroid, n_eff=self.n_eff, n_total=self.n_total, p_hi_c=self.p_hi_c,
                     level0_phase=self.level0_phase, alive=self.alive, s_h=self.s_h, recent_k=self.recent_k,
                     recent_k_raw=self.recent_k_raw, recent_v=self.recent_v, recent_pos=self.recent_pos,
                     recent_ends=self._recent_ends, alpha_k_raw=self.alpha_k_raw, alpha_v=self.alpha_v,
                     alpha_pos=self.alpha_pos, alpha_valid=self.alpha_valid, alpha_span_len=self._span_len,
                     alpha_span_closed=self._span_closed, alpha_nspans=self._span_count,
                     alpha_rowcount=self._row_count, alpha_count=self._alpha_count_dev)
        self._state = _lib.State(**{name: _lib.ptr(t) for name, t in views.items()})
        return self._state

    @contextlib.contextmanager
    def _semantic_update_context(self, updates, *, replay=False):
        """Record flushes into ``updates`` (replay=False) or apply its records (replay=True)."""
        previous = self._active_updates, self._replaying_updates
        self._active_updates, self._replaying_updates = updates, replay
        try:
            yield
        finally:
            self._active_updates, self._replaying_updates = previous

    def _update_signature(self, take: int):
        L = self._layout
        return (L.batch, L.groups, L.dim, L.clusters, L.levels, L.slots, L.recent_capacity, L.exact, L.span_cap,
                L.beta, L.dtype, L.eta, L.g0, L.lam, L.route, L.merge_passes, int(take), int(self.recent_count))

    def _flush_with_updates(self, take: int, record_op_log: bool, replay: bool) -> None:
        """One flush under an update context: record it, or replay its record without routing."""
        updates = self._active_updates
        key = (self._flush_cursor, int(take), int(self.recent_count))
        lib = _lib.lib()
        dev = self.level_k.device
        if self._replaying_updates:
            if not replay or key not in updates.flushes:
                if replay and any(k[0] < key[0] for k in updates.flushes):
                    raise RuntimeError("semantic update replay flushes are out of order")
                raise RuntimeError("missing semantic update record; rerouting is not allowed")
            signature, index, ready = updates.flushes[key]
            if signature != self._update_signature(take):
                raise RuntimeError("semantic update record does not match this flush/configuration")
            tape = updates.tensors[index]
            stream = torch.cuda.current_stream(dev)
            if ready is not None:
                stream.wait_event(ready)   # device-side wait only
            tape.record_stream(stream)
            self._ladder_epoch += 1
            state = self._state_struct()
            _lib.check(lib.logkv_flush_replay(
                ctypes.byref(self._layout), ctypes.byref(state), int(take), int(self.recent_count),
                ctypes.c_void_p(self._workspace.data_ptr()), self._workspace.numel(), ctypes.c_void_p(tape.data_ptr()),
                tape.numel(), ctypes.c_void_p(_lib.stream_ptr(dev))), "logkv_flush_replay")
            return
        if replay or key in updates.flushes:
            raise RuntimeError("duplicate or incorrectly bound semantic update recording")
        if not record_op_log:
            raise RuntimeError("semantic update recording requires record_op_log=True")
        nbytes = lib.logkv_tape_bytes(ctypes.byref(self._layout), int(take))
        tape = torch.empty(nbytes, dtype=torch.uint8, device=dev)
        self._ladder_epoch += 1
        state = self._state_struct()
        if self.kv_shard_group is not None:
            # The scores of this rank's groups, the span-part exchange, then the commit with the
            # record (which holds the ranks' common span choice: its replay needs no exchange).
            args = self._flush_args(take)
            world = self._gather_parts(args, take)
            _lib.check(lib.logkv_flush_commit_record(
                *args[:6], ctypes.c_void_p(self._span_gather.data_ptr()), world, 0, ctypes.c_void_p(tape.data_ptr()),
                tape.numel(), args[6]), "logkv_flush_commit_record")
        else:
            _lib.check(lib.logkv_flush_record(
                ctypes.byref(self._layout), ctypes.byref(state), int(take), int(self.recent_count),
                ctypes.c_void_p(self._workspace.data_ptr()), self._workspace.numel(),
                ctypes.c_void_p(tape.data_ptr()), tape.numel(), ctypes.c_void_p(_lib.stream_ptr(dev))),
                "logkv_flush_record")
        ready = torch.cuda.Event()
        ready.record(torch.cuda.current_stream(dev))
        index = updates.save(tape, owned=True)
        updates.flushes[key] = (self._update_signature(take), index, ready)

    # ------------------------------------------------------------------ op-log
    def begin_op_log(self) -> None:
        """Bind a fresh per-(batch, group) route log (the reference's begin_op_log, :2006-2028)."""
        cap = max(1, self.max_seq_length * 3)
        dev = self.level_count.device
        self.op_log = torch.zeros(self.batch_size, self.n_groups, cap, 4, device=dev, dtype=torch.int32)
        self.op_log_len = torch.zeros(self.batch_size, self.n_groups, device=dev, dtype=torch.int32)

    def take_op_log(self):
        """(log [B, G, max_len, 4], lengths [B, G]) as the reference's take_op_log (:2030-2038); synchronizes."""
        if getattr(self, "op_log", None) is None or getattr(self, "op_log_len", None) is None:
            return None, None
        lengths = self.op_log_len.clone()
        max_len = int(lengths.max().item()) if lengths.numel() else 0
        if max_len > self.op_log.size(2):
            raise RuntimeError("semantic LogKV op_log overflow")
        return self.op_log[:, :, :max_len].clone(), lengths

    def _append_op_log(self, take: int) -> None:
        """Append the rows of the flush just enqueued (same workspace) to the bound op-log."""
        if getattr(self, "op_log", None) is None:
            self.begin_op_log()
        _lib.check(_lib.lib().logkv_flush_oplog_append(
            ctypes.byref(self._layout), int(take), ctypes.c_void_p(self._workspace.data_ptr()),
            ctypes.c_void_p(self.op_log.data_ptr()), ctypes.c_void_p(self.op_log_len.data_ptr()),
            self.op_log.size(2), ctypes.c_void_p(_lib.stream_ptr(self.level_k.device))), "logkv_flush_oplog_append")

    def _route_decision_stream(self, take: int):
        """High-priority side stream ordered after the previous flush, or None.

        The decisions read the flushed window rows, the exact pool and the cluster state that
        the previous flush committed, and write only this cache's workspace; the rest of the
        flush returns to the caller's stream after them.  Only when every flushed row was
        already in the window at the end of the previous flush (rows appended since then keep
        the caller's stream), without profiling or KV-head sharding, and inside a CUDA-graph
        capture only when the previous flush was recorded in the same capture (the fork becomes
        a graph branch; an event of another capture or of eager work cannot be waited on there).
        """
        dev = self.level_k.device
        if (not self._route_overlap or dev.type != "cuda" or self._route_ready is None
                or self.semantic_unified_route
                or self.kv_shard_group is not None or self.profile_events is not None
                or take > self._route_ready_rows
                or self._route_ready_capture != _lib.capture_id(dev)):
            return None
        stream = self._ROUTE_STREAMS.get(dev)
        if stream is None:
            stream = self._ROUTE_STREAMS[dev] = torch.cuda.Stream(dev, priority=-1)
        stream.wait_event(self._route_ready)
        return stream

    def _route_mark_ready(self) -> None:
        """Record where the next flush's decisions may start (after this flush and its readers)."""
        dev = self.level_k.device
        if not self._route_overlap or dev.type != "cuda":
            self._route_ready = None
            return
        if self._route_ready is None:
            self._route_ready = torch.cuda.Event()
        self._route_ready.record(torch.cuda.current_stream(dev))
        self._route_ready_rows = self.recent_count
        self._route_ready_capture = _lib.capture_id(dev)

    def _flush_args(self, take: int):
        state = self._state_struct()
        return (ctypes.byref(self._layout), ctypes.byref(state), int(take), int(self.recent_count),
                ctypes.c_void_p(self._workspace.data_ptr()), self._workspace.numel(),
                ctypes.c_void_p(_lib.stream_ptr(self.level_k.device)))

    def _local_parts(self, take: int) -> torch.Tensor:
        """This rank's per-group span parts of a flush of ``take`` tokens (a workspace view)."""
        ptr, count = ctypes.POINTER(ctypes.c_float)(), ctypes.c_size_t()
        _lib.check(_lib.lib().logkv_flush_partials(ctypes.byref(self._layout), int(take),
                                                   ctypes.c_void_p(self._workspace.data_ptr()), ctypes.byref(ptr),
                                                   ctypes.byref(count)), "logkv_flush_partials")
        offset = ctypes.cast(ptr, ctypes.c_void_p).value - self._workspace.data_ptr()
        return self._workspace[offset:offset + 4 * count.value].view(torch.float32)

    def flush_device(self, take: int) -> None:
        """One device flush of the ``take`` oldest window tokens plus the window shift."""
        self._ladder_epoch += 1
        args = self._flush_args(take)
        if self.kv_shard_group is not None:
            self._sharded_flush(args, int(take))
            return
        side = self._route_decision_stream(int(take))
        if side is not None:
            lib = _lib.lib()
            _lib.check(lib.logkv_flush_decide(*args[:6], ctypes.c_void_p(side.cuda_stream)), "logkv_flush_decide")
            if self._route_done is None:
                self._route_done = torch.cuda.Event()
            self._route_done.record(side)
            torch.cuda.current_stream(self.level_k.device).wait_event(self._route_done)
            _lib.check(lib.logkv_flush_apply(*args), "logkv_flush_apply")
            return
        if self.profile_events is None:
            _lib.check(_lib.lib().logkv_flush(*args), "logkv_flush")
            return
        events = (ctypes.c_void_p * len(self.profile_events))(*[e.cuda_event for e in self.profile_events])
        _lib.check(_lib.lib().logkv_flush_profiled(*args, events, len(self.profile_events)), "logkv_flush_profiled")

    def _gather_parts(self, args, take: int) -> int:
        """Scores of this rank's groups and the all-gather of every rank's span parts into
        ``self._span_gather``; returns the rank count."""
        import torch.distributed as dist
        from .sharding import gather_span_parts
        _lib.check(_lib.lib().logkv_flush_scores(*args), "logkv_flush_scores")
        local = self._local_parts(take)
        world = dist.get_world_size(self.kv_shard_group)
        if self._span_gather is None or self._span_gather.numel() != world * local.numel():
            self._span_gather = torch.empty(world * local.numel(), dtype=torch.float32, device=self._workspace.device)
        gather_span_parts(local, self.kv_shard_group, out=self._span_gather)
        return world

    def _sharded_flush(self, args, take: int) -> None:
        """Scores of this rank's groups, all-gather of every rank's span parts, then the commit."""
        world = self._gather_parts(args, take)
        _lib.check(_lib.lib().logkv_flush_commit(*args[:6], ctypes.c_void_p(self._span_gather.data_ptr()), world,
                                                 args[6]), "logkv_flush_commit")

    def read_counters(self) -> dict:
        """Row counters accumulated by every flush of this cache (synchronizes)."""
        out = (ctypes.c_uint64 * len(_lib.COUNTERS))()
        _lib.check(_lib.lib().logkv_read_counters(ctypes.c_void_p(self._workspace.data_ptr()), out,
                                                  len(_lib.COUNTERS),
                                                  ctypes.c_void_p(_lib.stream_ptr(self.level_k.device))),
                   "logkv_read_counters")
        return dict(zip(_lib.COUNTERS, (int(x) for x in out)))

    def read_unified(self) -> dict:
        """Unified route: per-(batch, group) lane figures of the last flush (synchronizes): rounds,
        merges and live counts of the candidate and global passes, candidates, Ward merges."""
        if not self.semantic_unified_route:
            raise RuntimeError("read_unified applies to caches with semantic_unified_route=True")
        n = self.batch_size * self.n_groups * len(_lib.UNIFIED_WORDS)
        out = (ctypes.c_int32 * n)()
        _lib.check(_lib.lib().logkv_read_unified(ctypes.byref(self._layout), self.semantic_flush_granularity,
                                                 ctypes.c_void_p(self._workspace.data_ptr()), out, n,
                                                 ctypes.c_void_p(_lib.stream_ptr(self.level_k.device))),
                   "logkv_read_unified")
        words = np.frombuffer(out, dtype=np.int32).reshape(self.batch_size, self.n_groups, len(_lib.UNIFIED_WORDS))
        return {name: words[..., i].copy() for i, name in enumerate(_lib.UNIFIED_WORDS) if not name.startswith("unused")}

    def read_ties(self, clear: bool = True) -> list[dict]:
        """Near-tie log of this cache's flushes since the last clear (synchronizes).

        One dict per decision whose two best candidates (or value and threshold) were within a
        relative gap of 1e-6: kind, flush (0-based, counted since the cache was built), batch,
        group, cluster, index, first, second, gap, value (fields of logkv_tie_t).  Entries beyond
        the device log's 4096-entry capacity are only counted, in ``self.ties_dropped``.
        """
        cap = 4096
        out = (_lib.Tie * cap)()
        total = ctypes.c_int64(0)
        _lib.check(_lib.lib().logkv_read_ties(ctypes.c_void_p(self._workspace.data_ptr()), out, cap,
                                              ctypes.byref(total), int(clear),
                                              ctypes.c_void_p(_lib.stream_ptr(self.level_k.device))),
                   "logkv_read_ties")
        n = min(int(total.value), cap)
        self.ties_dropped = int(total.value) - n
        return [dict(kind=_lib.TIE_KINDS.get(e.kind, str(e.kind)), flush=e.flush, batch=e.batch, group=e.group,
                     cluster=e.cluster, index=e.index, first=e.first, second=e.second, gap=e.gap, value=e.value)
                for e in out[:n]]

    def read_status(self) -> int:
        out = ctypes.c_int32(0)
        _lib.check(_lib.lib().logkv_read_status(ctypes.c_void_p(self._workspace.data_ptr()), ctypes.byref(out),
                                                ctypes.c_void_p(_lib.stream_ptr(self.level_k.device))),
                   "logkv_read_status")
        return int(out.value)

    # ------------------------------------------------------------------ window
    def _positions(self, n: int, input_pos):
        """Absolute positions of the chunk's tokens as a [batch, n] int64 device tensor, or None for
        the consecutive positions token_count, token_count + 1, ... (written by the append kernel)."""
        dev = self.recent_pos.device
        if input_pos is None:
            return None
        if input_pos.dim() == 1:
            if input_pos.numel() != n:
                raise ValueError(f"input_pos length {input_pos.numel()} != chunk size {n}")
            return input_pos.to(device=dev, dtype=torch.int64).unsqueeze(0).expand(self.batch_size, -1)
        if input_pos.dim() == 2:
            if input_pos.shape != (self.batch_size, n):
                raise ValueError(f"input_pos shape {tuple(input_pos.shape)} != ({self.batch_size}, {n})")
            return input_pos.to(device=dev, dtype=torch.int64)
        raise ValueError(f"input_pos must be 1-D or 2-D, got shape {tuple(input_pos.shape)}")

    def add_recent(self, k, v, *, k_raw=None, input_pos=None, record_op_log=False, span_ends=None,
                   span_ends_device=None, **replay):
        """Append a chunk to the window; flush ``semantic_flush_granularity`` blocks on overflow.

        ``span_ends`` is the reference's host list of per-row boundary flags.
        ``span_ends_device`` (optional, uint8 [B, n] on the cache device) holds
        the same flags already on the device, so the call issues no host-to-device
        copy and can be captured in a CUDA graph.
        """
        replaying = any(v_ is not None for v_ in replay.values())
        chunk = self._check_chunk(k, v, k_raw, input_pos, span_ends, span_ends_device)
        take = None if replaying else self._chunk_flush_take(chunk[-1])
        if take is not None:
            # The one flush this chunk triggers, with the chunk written once after the shift.
            self._flush_chunk(chunk, take)
            if record_op_log:
                self._append_op_log(take)
            self._finish_flush(take)
            return
        self._append_window(*chunk)
        self.recent_count += chunk[-1]
        for take in self._pending_flushes():
            if self._active_updates is None and replaying:
                # As the reference's Alpha flush (log_kv_cache.py:5060-5061): an op-log alone cannot
                # replay an Alpha flush; the update tape can.
                raise RuntimeError("AlphaLogKV replay requires semantic_replay_updates; reranking is not allowed")
            if self._active_updates is not None:
                self._flush_with_updates(take, record_op_log, replaying or self._replaying_updates)
            else:
                self.flush_device(take)
            if record_op_log:
                self._append_op_log(take)
            self._finish_flush(take)

    def add_recent_deferred(self, k, v, *, k_raw=None, input_pos=None, span_ends=None, span_ends_device=None):
        """add_recent whose flush stops before the span choice, so that the caller can exchange many
        caches' span parts in one collective (``logkv_b200.sharding.BatchedFlush``); no reference
        counterpart.  Appends the chunk; when it makes the window overflow by one flush, runs the
        flush up to this cache's per-group span parts (``logkv_flush_scores``) and returns them (a
        [parts] float32 view of the workspace); ``commit_deferred`` must follow before any other
        call.  Returns None when the chunk flushes nothing."""
        if self._active_updates is not None:
            raise NotImplementedError("deferred flushes do not record or replay update tapes")
        if self._deferred_take is not None:
            raise RuntimeError("commit_deferred must follow add_recent_deferred")
        self._append_chunk(k, v, k_raw, input_pos, span_ends, span_ends_device)
        takes = list(self._pending_flushes())
        if not takes:
            return None
        if len(takes) > 1:
            raise NotImplementedError("a deferred chunk may overflow the window by one flush only")
        take = takes[0]
        self._ladder_epoch += 1
        args = self._flush_args(take)
        lib = _lib.lib()
        _lib.check(lib.logkv_flush_scores(*args), "logkv_flush_scores")
        self._deferred_take = take
        return self._local_parts(take)

    def commit_deferred(self, parts_all=None, ranks: int = 1, rank_stride: int = 0) -> None:
        """Finish the flush ``add_recent_deferred`` started: rank r's span parts of this cache at
        parts_all[r * rank_stride:] (float32 on the device; None with ranks == 1: this cache's own)."""
        take = self._deferred_take
        if take is None:
            raise RuntimeError("no deferred flush to commit")
        if ranks > 1 and parts_all is None:
            raise ValueError("the gathered span parts of every rank are needed")
        args = self._flush_args(take)
        ptr = ctypes.c_void_p(parts_all.data_ptr()) if parts_all is not None else None
        stride = int(rank_stride) if rank_stride else int(self._local_parts(take).numel())
        _lib.check(_lib.lib().logkv_flush_commit_strided(*args[:6], ptr, int(ranks), stride, args[6]),
                   "logkv_flush_commit_strided")
        self._deferred_take = None
        self._finish_flush(take)

    def _append_chunk(self, k, v, k_raw, input_pos, span_ends, span_ends_device) -> None:
        """Validation and the window write of add_recent (log_kv_cache.py:5668-5707)."""
        chunk = self._check_chunk(k, v, k_raw, input_pos, span_ends, span_ends_device)
        self._append_window(*chunk)
        self.recent_count += chunk[-1]

    def _chunk_flush_take(self, n: int):
        """The flush size when this chunk's add_recent is one flush of rows already in the window
        (logkv_flush_chunk's case: recent_count in [take, 2 take]), on the plain device path (no
        update tape, KV-head sharding or route overlap); else None."""
        if self._active_updates is not None or self.kv_shard_group is not None or self._route_overlap:
            return None
        c0, gran = self.recent_count, self.semantic_flush_granularity
        overflow = c0 + n - self.recent_size
        if overflow <= 0 or overflow > gran:
            return None
        return gran if gran <= c0 <= 2 * gran else None

    def _flush_chunk(self, chunk, take: int) -> None:
        """logkv_flush_chunk: the flush of the ``take`` oldest rows, then the kept rows and the
        chunk written to their places (same state as _append_window + flush_device)."""
        k, k_raw, v, positions, ends, n = chunk
        self._ladder_epoch += 1
        st, keep = self._chunk_struct(k, k_raw, v, positions, ends, n)
        args = self._flush_args(take)
        lib = _lib.lib()
        if self.profile_events is None:
            _lib.check(lib.logkv_flush_chunk(*args[:4], ctypes.byref(st), *args[4:]), "logkv_flush_chunk")
        else:
            events = (ctypes.c_void_p * len(self.profile_events))(*[e.cuda_event for e in self.profile_events])
            _lib.check(lib.logkv_flush_chunk_profiled(*args[:4], ctypes.byref(st), *args[4:], events,
                                                      len(self.profile_events)), "logkv_flush_chunk_profiled")
        del keep
        self.recent_count += n

    def _check_chunk(self, k, v, k_raw, input_pos, span_ends, span_ends_device):
        """Validation of add_recent (log_kv_cache.py:5668-5700): the chunk's rows, positions and
        span-end flags on the device, as (k, k_raw, v, positions, ends, n); counts the tokens."""
        if k_raw is None:
            raise ValueError("semantic LogKV add_recent requires pre-RoPE k_raw")
        n = k.size(2)
        if n > self.recent_size:
            raise ValueError(f"chunk size {n} exceeds recent_size {self.recent_size}")
        if k_raw.shape[:3] != k.shape[:3] or k_raw.size(-1) != self.k_dim:
            raise ValueError(f"k_raw shape {tuple(k_raw.shape)} does not match semantic cache shape")
        if span_ends is None or len(span_ends) != self.batch_size or any(len(r) != n for r in span_ends):
            raise ValueError("AlphaLogKV span boundaries must match the input batch and token count")
        positions = self._positions(n, input_pos)
        if self.token_count + n > self.max_seq_length:
            raise RuntimeError(f"LogStructuredKVCache: token overflow! token_count={self.token_count}, n={n}, "
                               f"max_seq_length={self.max_seq_length}.")
        if self.recent_count + n > self.recent_capacity:
            raise RuntimeError(f"semantic LogKV recent buffer overflow: recent_count={self.recent_count}, n={n}, "
                               f"capacity={self.recent_capacity}")
        self.token_count += n
        if span_ends_device is not None:
            ends = span_ends_device.to(device=self.recent_pos.device, dtype=torch.uint8).contiguous()
        else:
            host = torch.tensor(span_ends, dtype=torch.uint8)
            ends = self._ends_stage[:self.batch_size * n].view(self.batch_size, n)
            ends.copy_(host.pin_memory() if self.recent_pos.is_cuda else host, non_blocking=True)
        return k, k_raw, v, positions, ends, n

    def _pending_flushes(self):
        """Sizes of the flushes the window overflow needs (_semantic_add_recent :5708-5718)."""
        overflow = self.recent_count - self.recent_size
        if overflow <= 0:
            return
        gran = self.semantic_flush_granularity
        pending = gran * ((overflow + gran - 1) // gran)
        left = self.recent_count
        while pending > 0:
            take = min(gran, pending)
            if take > left:
                raise RuntimeError(f"semantic LogKV cannot flush {take} tokens from recent_count={left}")
            yield take
            left -= take
            pending -= take

    def _finish_flush(self, take: int) -> None:
        self._flush_cursor += 1
        self.recent_count -= take
        self._route_mark_ready()

    def _chunk_struct(self, k, k_raw, v, positions, ends, n: int):
        """(logkv_chunk_t, tensors it points into).  Rows must be in the storage dtype, contiguous
        along the head dim and 16-byte aligned; other inputs are made so first."""
        dt, dev = self.recent_k.dtype, self.recent_k.device
        esize = self.recent_k.element_size()

        def rows(t):
            if (t.dtype != dt or t.device != dev or t.stride(-1) != 1 or t.data_ptr() % 16
                    or any((st * esize) % 16 for st in t.stride()[:3])):
                t = t.to(device=dev, dtype=dt).contiguous()
            return t

        k, kr, v = rows(k), rows(k_raw), rows(v)
        c = _lib.Chunk()
        c.k, c.k_raw, c.v = k.data_ptr(), kr.data_ptr(), v.data_ptr()
        c.k_strides[:] = k.stride()[:3]
        c.k_raw_strides[:] = kr.stride()[:3]
        c.v_strides[:] = v.stride()[:3]
        if positions is not None:
            if positions.dtype != torch.int64 or positions.device != dev:
                positions = positions.to(device=dev, dtype=torch.int64)
            c.positions = positions.data_ptr()
            c.pos_strides[:] = positions.stride()
        c.pos0 = int(self.token_count - n)
        c.ends = ends.data_ptr()
        c.n = int(n)
        return c, (k, kr, v, positions, ends)

    def _append_window(self, k, k_raw, v, positions, ends, n: int) -> None:
        """The chunk into window rows [recent_count, recent_count + n) with one kernel
        (logkv_window_append)."""
        c, keep = self._chunk_struct(k, k_raw, v, positions, ends, n)
        state = self._state_struct()
        pos = ctypes.c_void_p(c.positions) if c.positions else None
        _lib.check(_lib.lib().logkv_window_append(
            ctypes.byref(self._layout), ctypes.byref(state), ctypes.c_void_p(c.k), c.k_strides,
            ctypes.c_void_p(c.k_raw), c.k_raw_strides, ctypes.c_void_p(c.v), c.v_strides, pos,
            c.pos_strides if c.positions else None, c.pos0, ctypes.c_void_p(c.ends), c.n, int(self.recent_count),
            ctypes.c_void_p(_lib.stream_ptr(self.recent_k.device))), "logkv_window_append")
        del keep

    # ------------------------------------------------------------------ read side
    def _semantic_attention_plan(self):
        """(physical_idx, anchors, M_s, valid) of the mid-anchor plan (log_kv_cache.py:5954-6007)."""
        from .attention import plan
        return plan(self)

    # ------------------------------------------------------------------ host mirrors (lazy, synchronizing)
    @property
    def alpha_count(self) -> int:
        return int(self._alpha_count_dev.item())

    @property
    def _semantic_counts(self):
        return self.level_count.long().tolist()

    @property
    def _semantic_alive(self):
        return self.alive.tolist()

    @property
    def _semantic_p_hi_c(self):
        return self.p_hi_c.tolist()

    @property
    def _semantic_n_total(self):
        return self.n_total.long().tolist()

    @property
    def _semantic_level0_phase(self):
        return self.level0_phase.long().tolist()

    @property
    def _semantic_current_segment(self):
        return self.current_segment.long().tolist()

    @property
    def _recent_pos_host(self):
        return self.recent_pos.tolist()

    @property
    def _recent_span_ends(self):
        return [[bool(x) for x in r] for r in self._recent_ends.tolist()]

    @property
    def _alpha_spans(self):
        lens, closed, count = self._span_len.tolist(), self._span_closed.tolist(), self._span_count.tolist()
        return [[(lens[b][i], bool(closed[b][i])) for i in range(count[b])] for b in range(self.batch_size)]

    @property
    def _alpha_positions(self):
        pos, rows = self.alpha_pos.tolist(), self._row_count.tolist()
        return [pos[b][:rows[b]] for b in range(self.batch_size)]

    def reset_parameters(self) -> None:
        """Empty cache: every buffer and mirror back to its constructor value."""
        i64max = torch.iinfo(torch.int64).max
        for name in ("recent_k", "recent_v", "recent_k_raw", "recent_pos", "alpha_k_raw", "alpha_v", "alpha_pos",
                     "alpha_valid", "level_k", "level_v", "level_w", "level_imp", "level_count", "pad_mask",
                     "level_sum_wp", "level_order", "centroid", "n_eff", "n_total", "current_segment",
                     "level0_phase", "alive"):
            getattr(self, name).zero_()
        self.level_p_lo.fill_(i64max)
        self.level_p_hi.fill_(-1)
        self.p_hi_c.fill_(-1)
        self.ward_cost.fill_(float("inf"))
        for t in (self._recent_ends, self._span_len, self._span_closed, self._span_count, self._row_count,
                  self._alpha_count_dev):
            t.zero_()
        self.token_count = 0
        self.recent_count = 0
        self._flush_cursor = 0
        self._route_ready = None
        self._deferred_take = None
        self._ladder_epoch += 1
