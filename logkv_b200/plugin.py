"""Operator-level plugin module: the reference's fused-kernel functions on sm_100a.

The reference resolves its fused kernels through ``_triton_updates()`` and
``_triton_route()`` (litgpt/log_kv_cache.py:339-354) and ``_triton_packer()``
(litgpt/log_kv_pack.py:18-24); each returns a module whose functions its
Python orchestration calls.  This module exports the same functions with the
same signatures, arguments and return values, implemented by the C ABI in
include/logkv_plugin.h (and include/logkv_attention.h for ``pack``):

  fill, merge_scatter, centroid, centroid_parallel, alpha_partition  (log_kv_updates_triton.py:79-328)
  attach_assign                                                      (log_kv_route_triton.py:894)
  pack                                                               (log_kv_pack_triton.py:95)

Results follow the reference's CPU order (feature sums left to right, no fused
multiply-adds), so they equal its CPU path; ``centroid_parallel`` is the same
ordered reduction.  The unified-route functions of log_kv_route_triton.py
(:546-838) are provided too, by include/logkv_unified.h:

  pair_distances, mirror, UnifiedReduce (single-pass rounds)

with the results of the reference's Torch reducer (_UnifiedReduceTorch).
"""
from __future__ import annotations

import ctypes

import torch

from . import _lib

_FIELDS = (0, 1, 2, 8, 9, 10, 11, 12)


class Rows(ctypes.Structure):
    _fields_ = [("k", ctypes.c_void_p), ("v", ctypes.c_void_p), ("w", ctypes.c_void_p), ("p_lo", ctypes.c_void_p),
                ("p_hi", ctypes.c_void_p), ("sum_wp", ctypes.c_void_p), ("order", ctypes.c_void_p),
                ("pad", ctypes.c_void_p), ("kv_dtype", ctypes.c_int32)]


class Partition(ctypes.Structure):
    _fields_ = [(n, ctypes.c_void_p) for n in ("k", "v", "pos", "indices", "exact_k", "exact_v", "exact_pos",
                                                "exact_valid", "archive_k", "archive_v", "archive_pos")] + \
               [(n, ctypes.c_int32) for n in ("batch", "groups", "tokens", "exact", "archive", "dk", "dv", "dtype")]


class Attach(ctypes.Structure):
    _fields_ = [("x", ctypes.c_void_p), ("x_stride_b", ctypes.c_int64), ("x_stride_g", ctypes.c_int64),
                ("x_stride_t", ctypes.c_int64), ("positions", ctypes.c_void_p), ("pos_stride_b", ctypes.c_int64),
                ("order", ctypes.c_void_p), ("counts", ctypes.c_void_p), ("centroid", ctypes.c_void_p),
                ("alive", ctypes.c_void_p), ("p_hi", ctypes.c_void_p), ("s_h", ctypes.c_void_p),
                ("out", ctypes.c_void_p)] + \
               [(n, ctypes.c_int32) for n in ("batch", "groups", "tokens", "clusters", "dim", "dtype")] + \
               [("eta", ctypes.c_float), ("g0", ctypes.c_float), ("lam", ctypes.c_float)]


_bound = False


class Unified(ctypes.Structure):
    _fields_ = [(n, ctypes.c_void_p) for n in ("dist", "mu", "mass", "limits", "status", "alive", "radius",
                                                "packed", "merges", "stuck", "trace")] + \
               [(n, ctypes.c_int32) for n in ("lanes", "size", "dim", "target")]


def _lib_plugin():
    global _bound
    lib = _lib.lib()
    if not _bound:
        P, v, i64, i32 = ctypes.POINTER, ctypes.c_void_p, ctypes.c_int64, ctypes.c_int32
        lib.logkv_fill.restype = ctypes.c_int
        lib.logkv_fill.argtypes = [P(Rows), P(Rows), v, v, i64, i32, i32, v]
        lib.logkv_merge_scatter.restype = ctypes.c_int
        lib.logkv_merge_scatter.argtypes = [P(Rows), P(Rows), v, i64, v, v, i64, v, i64, v, v, i64, P(Rows), v, i64,
                                            v, i32, i32, i32, v]
        lib.logkv_centroid.restype = ctypes.c_int
        lib.logkv_centroid.argtypes = [v, i32, i32, v, v, v, i64, i64, i64, v, v]
        lib.logkv_alpha_partition.restype = ctypes.c_int
        lib.logkv_alpha_partition.argtypes = [P(Partition), v]
        lib.logkv_attach_assign.restype = ctypes.c_int
        lib.logkv_attach_assign.argtypes = [P(Attach), v]
        lib.logkv_pair_distances.restype = ctypes.c_int
        lib.logkv_pair_distances.argtypes = [v, v, i32, i32, v]
        lib.logkv_mirror.restype = ctypes.c_int
        lib.logkv_mirror.argtypes = [v, i32, i32, v]
        lib.logkv_unified_init.restype = ctypes.c_int
        lib.logkv_unified_init.argtypes = [P(Unified), v]
        lib.logkv_unified_step.restype = ctypes.c_int
        lib.logkv_unified_step.argtypes = [P(Unified), v]
        _bound = True
    return lib


def _stream(t: torch.Tensor) -> ctypes.c_void_p:
    return ctypes.c_void_p(_lib.stream_ptr(t.device))


def _dtype(t: torch.Tensor) -> int:
    if t.dtype not in _lib.DTYPE_CODES:
        raise ValueError(f"unsupported dtype {t.dtype} (float32 or bfloat16)")
    return _lib.DTYPE_CODES[t.dtype]


def _i64(t: torch.Tensor) -> torch.Tensor:
    return t.to(torch.int64).contiguous()


def _rows(fields) -> Rows:
    """Rows struct of a reference 13-field tuple (fields 0, 1, 2, 8-12, contiguous)."""
    f = [fields[i] for i in _FIELDS]
    for t in f:
        if not t.is_contiguous():
            raise ValueError("ladder field views must be contiguous")
    if f[7].dtype != torch.bool or f[2].dtype != torch.float32 or any(t.dtype != torch.int64 for t in f[3:7]):
        raise ValueError("ladder fields must be (K, V, w float32, p_lo/p_hi/sum_wp/order int64, pad bool)")
    if f[0].dtype != f[1].dtype:
        raise ValueError("K and V fields must share a dtype")
    return Rows(*[_lib.ptr(t) for t in f], _dtype(f[0]))


def fill(fields, stage, src, dst):
    """Copy staged rows ``stage[src]`` into ``fields[dst]`` (log_kv_updates_triton.py:79-88)."""
    n = dst.numel()
    if not n:
        return
    src, dst = _i64(src), _i64(dst)
    _lib.check(_lib_plugin().logkv_fill(ctypes.byref(_rows(fields)), ctypes.byref(_rows(stage)), src.data_ptr(),
                                        dst.data_ptr(), n, fields[0].size(1), fields[1].size(1), _stream(dst)),
               "logkv_fill")


def merge_scatter(fields, stage, si, gi, pi, vi, dst, clear, *, beta_lengths=None, beta_cuts=None, beta_layout=None):
    """Merge pool pairs (or Beta groups) into a carry and scatter survivors (log_kv_updates_triton.py:176-220).

    Returns the 13-field carry tuple (float32 K/V, None for the unused fields),
    plus the uint8 Beta cuts when ``beta_lengths`` is given.
    """
    dev = fields[0].device
    pairs, survivors = pi.numel() // 2, vi.numel()
    n = pairs + survivors
    f = [fields[i] for i in _FIELDS]
    out = tuple(torch.empty((n, *x.shape[1:]), device=dev, dtype=torch.float32 if i < 2 else x.dtype)
                for i, x in enumerate(f))
    si, gi, pi, vi, dst, clear = (_i64(t) for t in (si, gi, pi, vi, dst, clear))
    layout_ptr, ngroups, cuts_ptr, mode = None, 0, None, 0
    if beta_lengths is not None:
        if sum(int(x) for x in beta_lengths) != pi.numel():
            raise ValueError("Beta lane lengths must cover the compaction input")
        if beta_layout is None:
            rows = []
            base = 0
            for length in beta_lengths:
                length = int(length)
                if length < 0 or length % 2:
                    raise ValueError("Beta compaction requires even nonnegative lane lengths")
                for off in range(0, length, 4):
                    rows.append((base + off, min(4, length - off), (base + off) // 2))
                base += length
            beta_layout = torch.tensor(rows, dtype=torch.int64, device=dev).reshape(-1, 3)
        expected = sum((int(x) + 3) // 4 for x in beta_lengths)
        if (beta_layout.ndim != 2 or beta_layout.shape[1] != 3 or beta_layout.dtype != torch.int64
                or beta_layout.device != pi.device or not beta_layout.is_contiguous() or len(beta_layout) != expected):
            raise ValueError("Beta layout does not match the compaction lanes")
        replay = beta_cuts is not None
        if not replay:
            beta_cuts = torch.empty(len(beta_layout), dtype=torch.uint8, device=dev)
        elif beta_cuts.shape != (len(beta_layout),) or beta_cuts.dtype != torch.uint8 or beta_cuts.device != pi.device:
            raise ValueError("recorded Beta cuts do not match the compaction layout")
        layout_ptr, ngroups, cuts_ptr, mode = beta_layout.data_ptr(), len(beta_layout), beta_cuts.data_ptr(), 2 if replay else 1
    out_rows = Rows(*[t.data_ptr() for t in out], _lib.DTYPE_CODES[torch.float32])
    ptr = lambda t: t.data_ptr() if t.numel() else None  # noqa: E731
    _lib.check(_lib_plugin().logkv_merge_scatter(
        ctypes.byref(_rows(fields)), ctypes.byref(_rows(stage)), ptr(si), si.numel(), ptr(gi), ptr(pi), pi.numel(),
        ptr(vi), survivors, ptr(dst), ptr(clear), clear.numel(), ctypes.byref(out_rows), layout_ptr, ngroups, cuts_ptr,
        mode, fields[0].size(1), fields[1].size(1), _stream(fields[0])), "logkv_merge_scatter")
    carry = [None] * 13
    for i, x in zip(_FIELDS, out):
        carry[i] = x[:pairs]
    return tuple(carry) if beta_lengths is None else (tuple(carry), beta_cuts)


def centroid(k, mu, n_eff, metadata, start, count, *, token_tile=1):
    """Ordered centroid updates of runs [start, start + count) (log_kv_updates_triton.py:268-278)."""
    if not count:
        return
    if mu.dtype != torch.float32 or n_eff.dtype != torch.float32 or not mu.is_contiguous():
        raise ValueError("centroid state must be contiguous float32")
    k = k.contiguous()
    meta = _i64(metadata)
    scratch = torch.empty(count * (k.size(1) + 1), dtype=torch.float32, device=k.device)
    _lib.check(_lib_plugin().logkv_centroid(k.data_ptr(), _dtype(k), k.size(1), mu.data_ptr(), n_eff.data_ptr(),
                                            meta.data_ptr(), meta.size(1), int(start), int(count), scratch.data_ptr(),
                                            _stream(k)), "logkv_centroid")


def centroid_parallel(k, mu, n_eff, metadata, start, count):
    """Same as ``centroid`` (the ordered reduction is already parallel over runs and features)."""
    centroid(k, mu, n_eff, metadata, start, count)


def alpha_partition(k, v, pos, indices, exact):
    """Copy kept rows into the exact pool and return the archived rows (log_kv_updates_triton.py:313-328)."""
    ek, ev, ep, valid = exact
    b, g, n, dk = k.shape
    p, a, dv = ek.size(2), indices.size(1) - ek.size(2), v.size(-1)
    k, v, pos, idx = k.contiguous(), v.contiguous(), _i64(pos), _i64(indices)
    ak, av = k.new_empty((b, g, a, dk)), v.new_empty((b, g, a, dv))
    ap = pos.new_empty((b, a))
    args = Partition(k.data_ptr(), v.data_ptr(), pos.data_ptr(), idx.data_ptr(), _lib.ptr(ek), _lib.ptr(ev),
                     _lib.ptr(ep), _lib.ptr(valid), ak.data_ptr() if a else None, av.data_ptr() if a else None,
                     ap.data_ptr() if a else None, b, g, n, p, a, dk, dv, _dtype(k))
    _lib.check(_lib_plugin().logkv_alpha_partition(ctypes.byref(args), _stream(k)), "logkv_alpha_partition")
    return ak, av, ap


def attach_assign(k_raw, positions, order, counts, centroid, alive, p_hi, s_h, eta, g0, lam):
    """Final attach cluster per token, int8 [B, G, T] in position order, no new clusters (route_triton.py:894)."""
    n_batch, n_groups, tokens, dim = k_raw.shape
    if k_raw.stride(-1) != 1:
        k_raw = k_raw.contiguous()
    if positions.stride(-1) != 1:
        positions = positions.contiguous()
    positions = positions if positions.dtype == torch.int64 else positions.to(torch.int64)
    out = torch.full((n_batch, n_groups, tokens), -1, dtype=torch.int8, device=k_raw.device)
    mu = centroid.float().contiguous()
    sh = s_h.float().contiguous()
    alive_u8 = alive.contiguous().view(torch.uint8) if alive.dtype == torch.bool else alive.to(torch.uint8).contiguous()
    phi, order, counts = _i64(p_hi), _i64(order), _i64(counts)
    args = Attach(k_raw.data_ptr(), k_raw.stride(0), k_raw.stride(1), k_raw.stride(2), positions.data_ptr(),
                  positions.stride(0), order.data_ptr(), counts.data_ptr(), mu.data_ptr(), alive_u8.data_ptr(),
                  phi.data_ptr(), sh.data_ptr(), out.data_ptr(), n_batch, n_groups, tokens, centroid.size(2), dim,
                  _dtype(k_raw), float(eta), float(g0), float(lam))
    _lib.check(_lib_plugin().logkv_attach_assign(ctypes.byref(args), _stream(k_raw)), "logkv_attach_assign")
    return out


def pack(cache, plan, k, v, dim, buffers=None, skip_pooled=False, recent_start=0):
    """Packed K/V with the mass coordinate (log_kv_pack_triton.py:95), bit for bit with the torch packer."""
    from .attention import pack_mid_kv
    return pack_mid_kv(cache, plan, k, v, dim, buffers=buffers, skip_pooled=skip_pooled, recent_start=recent_start)


# ------------------------------------------------------------------------------------------ unified route
def _f32(t: torch.Tensor, what: str) -> torch.Tensor:
    if t.dtype != torch.float32 or not t.is_cuda or not t.is_contiguous():
        raise ValueError(f"{what} must be a contiguous float32 CUDA tensor")
    return t


def pair_distances(gram, norm):
    """Contiguous FP32 Gram products [L, M, M] -> symmetric squared distances, in place
    (log_kv_route_triton.py:585-607): max((n_i + n_j) - 2 G_ij, 0) from the upper triangle."""
    _f32(gram, "gram")
    norm = norm.contiguous()
    _f32(norm, "norm")
    lanes, size = gram.shape[:2]
    _lib.check(_lib_plugin().logkv_pair_distances(ctypes.c_void_p(gram.data_ptr()), ctypes.c_void_p(norm.data_ptr()),
                                                  lanes, size, _stream(gram)), "logkv_pair_distances")
    return gram


def mirror(dist):
    """Make [L, M, M] exactly symmetric (log_kv_route_triton.py:546-553), in place."""
    _f32(dist, "dist")
    lanes, size = dist.shape[:2]
    _lib.check(_lib_plugin().logkv_mirror(ctypes.c_void_p(dist.data_ptr()), lanes, size, _stream(dist)),
               "logkv_mirror")
    return dist


class UnifiedReduce:
    """Device state of the incremental Ward rounds (log_kv_route_triton.py:610-838).

    Same constructor and methods as the reference's ``UnifiedReduce``: ``step(round_)`` queues
    one round and returns the per-lane active flags (int32, on the device), ``status`` holds
    (active, live count) per lane for the host to poll, ``limit_live`` is accepted (it only
    narrows launch grids in the reference; results do not depend on it), and ``finish()`` reads
    back (traces per lane [n, 2] int64, alive [L, M] bool, stuck [L] bool).  ``dist``, ``mu`` and
    ``mass`` are updated in place.  Only single-pass rounds: ``passes > 1`` (frozen-centre
    sweeps) raises NotImplementedError.
    """

    def __init__(self, dist, mu, mass, count, limits, target, passes=1):
        if int(passes) != 1:
            raise NotImplementedError("frozen-centre sweeps (passes > 1) are not implemented by logkv_b200")
        self.dist, self.mu, self.mass = _f32(dist, "dist"), _f32(mu, "mu"), _f32(mass, "mass")
        self.limits = None if limits is None else _f32(limits.contiguous(), "limits")
        lanes, size = mass.shape
        dev = mass.device
        self.target = int(target)
        self.status = torch.stack((torch.zeros(lanes, dtype=torch.int32, device=dev),
                                   count.to(device=dev, dtype=torch.int32)))
        self.active, self.count = self.status.unbind(0)
        self.alive = torch.zeros((lanes, size), dtype=torch.uint8, device=dev)
        self.radius = torch.zeros((lanes, size), dtype=torch.float32, device=dev)
        self.packed = torch.zeros((lanes, size), dtype=torch.int64, device=dev)
        self.merges = torch.zeros(lanes, dtype=torch.int32, device=dev)
        self.stuck = torch.zeros(lanes, dtype=torch.uint8, device=dev)
        self.trace = torch.zeros((lanes, size, 2), dtype=torch.int32, device=dev)
        self._u = Unified(*[ctypes.c_void_p(t.data_ptr()) if t is not None else None
                            for t in (self.dist, self.mu, self.mass, self.limits, self.status, self.alive,
                                      self.radius, self.packed, self.merges, self.stuck, self.trace)],
                          lanes, size, mu.size(-1), self.target)
        _lib.check(_lib_plugin().logkv_unified_init(ctypes.byref(self._u), _stream(mass)), "logkv_unified_init")

    def limit_live(self, count):
        """Accepted for interface parity; launch sizes here do not depend on a live bound."""
        return None

    def step(self, round_=None):
        _lib.check(_lib_plugin().logkv_unified_step(ctypes.byref(self._u), _stream(self.mass)), "logkv_unified_step")
        return self.active

    def finish(self):
        merges = self.merges.cpu().numpy()
        trace = self.trace.cpu().numpy().astype("int64")
        alive = self.alive.cpu().numpy().astype(bool)
        stuck = self.stuck.cpu().numpy().astype(bool)
        return [trace[lane, :n] for lane, n in enumerate(merges)], alive, stuck
