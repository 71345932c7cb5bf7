"""Read side of the cache: mid-anchor plan, packing and slot attention on the GPU.

Mirrors the reference's functions for the in-scope configuration (mid anchors,
first order) with the same names, arguments and errors:

  plan(cache)                     LogStructuredKVCache._semantic_attention_plan  (log_kv_cache.py:5954-6007)
  pack_mid_kv(cache, plan, ...)   log_kv_pack.pack_mid_kv                         (log_kv_pack.py:114-131)
  log_kv_chunk_attention(...)     log_kv_cache.log_kv_chunk_attention             (log_kv_cache.py:6802-6864)

Everything runs through the C ABI of ``liblogkv_b200.so`` (include/logkv_attention.h);
there is no CPU path.  The packed frozen prefix (merged slots rotated at their mid
anchors, then the exact pool) only changes when a flush rewrites the ladder, so it
is rebuilt on the device once per flush and reused by every attention call until
the next one: the reference's ``reuse_prefix`` decode workspace, made the default.
The kernels are forward-only.
"""
from __future__ import annotations

import ctypes

import torch

from . import _lib

# Query rows (heads per group x query tokens) one decode-kernel launch covers; bf16 chunks
# with more rows go to the chunk kernel in a single launch.
_MAX_QUERY_ROWS = {torch.bfloat16: 16, torch.float32: 8}


class _ReadState:
    """Device buffers of the plan, the packed prefix and the attention scratch of one cache."""

    def __init__(self, cache):
        dev = cache.level_k.device
        B, G = cache.batch_size, cache.n_groups
        cap = cache.K_max * cache.L_alloc * cache.B_prime
        P = cache.alpha_exact_tokens
        i32, i64 = dict(dtype=torch.int32, device=dev), dict(dtype=torch.int64, device=dev)
        self.cap = cap
        self.idx = torch.zeros(B, G, cap, **i64)
        self.anchor = torch.zeros(B, G, cap, **i64)
        self.valid = torch.zeros(B, G, cap, dtype=torch.uint8, device=dev)
        self.width = torch.zeros(B, G, **i32)
        self.width_max = torch.zeros(1, **i32)
        self.vslot = torch.zeros(B, G, cap, **i32)
        self.vanchor = torch.zeros(B, G, cap, **i64)
        self.nvalid = torch.zeros(B, G, **i32)
        self.exact_rows = torch.zeros(B, max(P, 1), **i32)
        self.nexact = torch.zeros(B, **i32)
        self.capacity = cap + P
        self.pk = torch.zeros(B, G, self.capacity, cache.k_dim, dtype=cache.level_k.dtype, device=dev)
        self.pv = torch.zeros(B, G, self.capacity, cache.v_dim, dtype=cache.level_v.dtype, device=dev)
        self.mass = torch.zeros(B, G, self.capacity, dtype=torch.float32, device=dev)
        self.length = torch.zeros(B, G, **i32)
        self.status = torch.zeros(1, **i32)
        self.epoch = -1
        self.workspaces: dict = {}

    def plan_struct(self, full: bool) -> _lib.Plan:
        p = lambda t: t.data_ptr()  # noqa: E731
        return _lib.Plan(p(self.idx) if full else None, p(self.anchor) if full else None,
                         p(self.valid) if full else None, p(self.width), p(self.width_max), p(self.vslot),
                         p(self.vanchor), p(self.nvalid), p(self.exact_rows), p(self.nexact))

    def prefix_struct(self) -> _lib.Prefix:
        return _lib.Prefix(self.pk.data_ptr(), self.pv.data_ptr(), self.mass.data_ptr(), self.length.data_ptr(),
                           self.capacity)

    def workspace(self, cache, heads: int, q_tokens: int) -> torch.Tensor:
        key = (heads, q_tokens)
        ws = self.workspaces.get(key)
        if ws is None:
            n = _lib.lib().logkv_attention_workspace_bytes(ctypes.byref(_structs(cache)[0]), heads, q_tokens,
                                                           self.capacity)
            if not n:
                raise ValueError(f"attention shape outside the supported range (heads={heads}, tokens={q_tokens})")
            ws = torch.zeros(n, dtype=torch.uint8, device=cache.level_k.device)
            self.workspaces[key] = ws
        return ws


class _ForeignCache:
    """Layout and state structs for a cache object that only has the reference's buffers.

    The reference's own ``LogStructuredKVCache`` on a CUDA device registers the same
    buffer names, shapes and dtypes (log_kv_cache.py:907-1122); the read-side kernels
    use only those.  Fields the read side never touches point at one small dummy buffer.
    """

    def __init__(self, cache):
        dev = cache.level_k.device
        self.dummy = torch.zeros(64, dtype=torch.int64, device=dev)
        self.alpha_count = torch.zeros(1, dtype=torch.int32, device=dev)
        B, G = cache.batch_size, cache.n_groups
        self.layout = _lib.Layout(B, G, cache.k_dim, cache.K_max, cache.L_alloc, cache.B_prime,
                                  cache.recent_k.size(2), cache.alpha_exact_tokens, 1, 0,
                                  _lib.DTYPE_CODES[cache.level_k.dtype], 1.0, 1.0, 1.0)

    def state(self, cache) -> _lib.State:
        self.alpha_count.fill_(int(cache.alpha_count))
        d = self.dummy.data_ptr()
        views = dict(level_k=cache.level_k, level_v=cache.level_v, level_w=cache.level_w,
                     level_sum_wp=cache.level_sum_wp, level_count=cache.level_count, recent_k=cache.recent_k,
                     recent_v=cache.recent_v, alpha_k_raw=cache.alpha_k_raw, alpha_v=cache.alpha_v,
                     alpha_pos=cache.alpha_pos, alpha_valid=cache.alpha_valid, alpha_count=self.alpha_count)
        ptrs = {name: d for name in _lib.STATE_FIELDS}
        ptrs.update({name: _lib.ptr(t) for name, t in views.items()})
        return _lib.State(**ptrs)


def _structs(cache):
    """(layout, state) of a logkv_b200 cache, or of any cache with the reference's buffers."""
    if hasattr(cache, "_state_struct"):
        return cache._layout, cache._state_struct()
    fc = getattr(cache, "_b200_foreign", None)
    if fc is None:
        fc = _ForeignCache(cache)
        cache._b200_foreign = fc
    return fc.layout, fc.state(cache)


def _read_state(cache) -> _ReadState:
    rs = getattr(cache, "_read", None)
    if rs is None:
        rs = _ReadState(cache)
        cache._read = rs
    return rs


def _rope(cache) -> _lib.Rope:
    cos, sin = cache.cos_cache, cache.sin_cache
    if cos.dtype not in _lib.DTYPE_CODES or sin.dtype != cos.dtype:
        raise ValueError("cos_cache/sin_cache must both be float32 or bfloat16")
    if cos.dim() != 2 or cos.shape != sin.shape:
        raise ValueError(f"cos_cache/sin_cache must be 2-D and equal in shape, got {cos.shape} and {sin.shape}")
    if cache.rope_n_elem and cos.size(1) != cache.rope_n_elem:
        raise ValueError("cos_cache width must equal rope_n_elem")
    return _lib.Rope(_lib.ptr(cos.contiguous()), _lib.ptr(sin.contiguous()), cos.size(0), cache.rope_n_elem,
                     _lib.DTYPE_CODES[cos.dtype])


def _stream(cache) -> ctypes.c_void_p:
    return ctypes.c_void_p(_lib.stream_ptr(cache.level_k.device))


def _run_plan(cache, full: bool) -> _ReadState:
    rs = _read_state(cache)
    layout, state = _structs(cache)
    plan = rs.plan_struct(full)
    _lib.check(_lib.lib().logkv_attention_plan(ctypes.byref(layout), ctypes.byref(state), ctypes.byref(plan),
                                               _stream(cache)), "logkv_attention_plan")
    return rs


def refresh_prefix(cache) -> _ReadState:
    """Plan and pack the frozen prefix when a flush has changed the ladder since the last pack."""
    rs = _read_state(cache)
    epoch = getattr(cache, "_ladder_epoch", None)   # None: a foreign cache, repack every call
    if epoch is not None and rs.epoch == epoch:
        return rs
    _run_plan(cache, full=False)
    layout, state = _structs(cache)
    plan, rope, pre = rs.plan_struct(False), _rope(cache), rs.prefix_struct()
    _lib.check(_lib.lib().logkv_pack_prefix(ctypes.byref(layout), ctypes.byref(state), ctypes.byref(plan),
                                            ctypes.byref(rope), ctypes.byref(pre), rs.status.data_ptr(),
                                            _stream(cache)), "logkv_pack_prefix")
    rs.epoch = epoch if epoch is not None else -1
    return rs


def plan(cache):
    """(physical_idx, anchors, M_s, valid), each [B, G, width] (log_kv_cache.py:5979-6007).

    Reads the plan width back to the host (one synchronization), as the
    reference's plan reads its host count mirror.
    """
    rs = _run_plan(cache, full=True)
    width = int(rs.width_max.item())
    idx = rs.idx[..., :width].clone()
    anchors = rs.anchor[..., :width].clone()
    valid = rs.valid[..., :width].bool()
    return idx, anchors, torch.ones_like(anchors), valid


def _check_kv(cache, k, v, name="k"):
    if k.dim() != 4 or k.shape[:2] != (cache.batch_size, cache.n_groups) or k.size(-1) != cache.k_dim:
        raise ValueError(f"{name} must be [B, G, T, {cache.k_dim}], got {tuple(k.shape)}")
    if v.shape[:3] != k.shape[:3] or v.size(-1) != cache.v_dim:
        raise ValueError(f"v shape {tuple(v.shape)} does not match k {tuple(k.shape)}")
    if k.dtype != cache.level_k.dtype or v.dtype != cache.level_k.dtype:
        raise ValueError(f"k/v dtype must be the cache dtype {cache.level_k.dtype}")


def pack_mid_kv(cache, plan_, k, v, dim, *, backend=None, buffers=None, skip_pooled=False, recent_start=0):
    """Final padded K/V with the mass/mask coordinate (log_kv_pack.py:27-72, :114-131), bit for bit."""
    backend = cache.semantic_pack_backend if backend is None else backend
    if backend not in ("auto", "torch", "triton"):
        raise ValueError("packing backend must be 'auto', 'torch' or 'triton'")
    if cache.semantic_anchor_mode != "mid":
        raise ValueError("pack_mid_kv requires semantic_anchor_mode='mid'")
    if buffers is None and (skip_pooled or recent_start):
        raise ValueError("skip_pooled and recent_start require reusable buffers")
    _check_kv(cache, k, v)
    if torch.is_grad_enabled() and (k.requires_grad or v.requires_grad):
        raise NotImplementedError("logkv_b200 packing is forward-only")
    if dim < max(cache.k_dim + 1, cache.v_dim):
        raise ValueError(f"dim {dim} too small for k_dim {cache.k_dim} + 1 and v_dim {cache.v_dim}")
    width = plan_[0].size(-1)
    rs = _run_plan(cache, full=True)
    exact, recent, T = cache.alpha_count, cache.recent_count, k.size(2)
    length = width + exact + recent + T
    shape = (cache.batch_size, cache.n_groups, length, dim)
    if buffers is None:
        ka = torch.empty(shape, dtype=k.dtype, device=k.device)
        va = torch.empty(shape, dtype=v.dtype, device=v.device)
    else:
        ka, va = (buf[:, :, :length] for buf in buffers)
        if not ka.is_contiguous():
            raise ValueError("reusable pack buffers must be contiguous in their first `length` rows")
    kc, vc = k.contiguous(), v.contiguous()
    layout, state = _structs(cache)
    plan_s, rope = rs.plan_struct(True), _rope(cache)
    _lib.check(_lib.lib().logkv_pack_mid(
        ctypes.byref(layout), ctypes.byref(state), ctypes.byref(plan_s), ctypes.byref(rope), width, exact,
        recent, kc.data_ptr(), vc.data_ptr(), T, ka.data_ptr(), va.data_ptr(), dim, int(bool(skip_pooled)),
        int(recent_start), rs.status.data_ptr(), _stream(cache)), "logkv_pack_mid")
    return ka, va


def query_extra(scale: float, dtype: torch.dtype) -> float:
    """``1/scale`` as the query dtype stores it (log_kv_cache.py:6459-6460)."""
    return float(torch.tensor(1.0 / scale, dtype=dtype))


def log_kv_chunk_attention(cache, q_b, k_b, v_b, scale, second_order_scale=1.0, attention_plan=None, *,
                           causal_tail=None, reuse_prefix=False, out=None):
    """One streaming attention step without committing the chunk (log_kv_cache.py:6802-6864).

    [frozen cache state (fully visible)] + [current chunk (lower-right causal)].
    The cache holds no second-order statistics, so ``second_order_scale`` has
    no effect, as in the reference.  ``attention_plan`` may be passed for API
    compatibility; the device plan is derived from the same ladder state.
    """
    causal_tail = q_b.size(2) if causal_tail is None else causal_tail
    if causal_tail and causal_tail != q_b.size(2):
        raise ValueError("causal_tail must equal query length or be zero")
    _check_kv(cache, k_b, v_b, "k_b")
    B, H, T, kd = q_b.shape
    if B != cache.batch_size or kd != cache.k_dim or q_b.dtype != cache.level_k.dtype:
        raise ValueError(f"q_b must be [B={cache.batch_size}, H, T, {cache.k_dim}] in the cache dtype")
    Tk = k_b.size(2)
    if T != Tk and (causal_tail or T > Tk):
        raise ValueError("q_b and k_b must cover the same tokens (fewer queries only with causal_tail=0)")
    G = cache.n_groups
    if H % G:
        raise ValueError(f"query heads {H} must be a multiple of KV groups {G}")
    if torch.is_grad_enabled() and any(t.requires_grad for t in (q_b, k_b, v_b)):
        raise NotImplementedError("logkv_b200 attention is forward-only")
    rs = refresh_prefix(cache)
    rf = H // G
    rows = _MAX_QUERY_ROWS[q_b.dtype]
    if rf > rows or rf & (rf - 1):
        raise ValueError(f"{rf} query heads per KV group: must be a power of two <= {rows}")
    if q_b.dtype == torch.bfloat16 and rf * T > rows and cache.k_dim <= 128 and rf <= 8:
        step = T                    # one launch of the chunk kernel
    else:
        step = 1
        while 2 * step * rf <= rows and 2 * step <= T:
            step *= 2
    q, k, v = q_b.contiguous(), k_b.contiguous(), v_b.contiguous()
    if out is None:
        out = torch.empty(B, H, T, cache.v_dim, dtype=q.dtype, device=q.device)
    layout, state = _structs(cache)
    pre = rs.prefix_struct()
    qx = query_extra(scale, q.dtype)
    t0 = 0
    while t0 < T:               # query blocks: the whole chunk, or powers of two of at most `step`
        n = step
        while n > T - t0:
            n //= 2
        ws = rs.workspace(cache, H, n)
        args = _lib.AttentionArgs(q.data_ptr(), k.data_ptr(), v.data_ptr(), out.data_ptr(), H, Tk, t0, n,
                                  int(cache.recent_count), int(bool(causal_tail)), float(scale), qx, T)
        _lib.check(_lib.lib().logkv_attention(ctypes.byref(layout), ctypes.byref(state), ctypes.byref(pre),
                                              ctypes.byref(args), ws.data_ptr(), ws.numel(), _stream(cache)),
                   "logkv_attention")
        t0 += n
    return out
