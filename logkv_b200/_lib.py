"""ctypes binding of the in-tree C-ABI library ``liblogkv_b200.so``.

The library is the product: there is no CPU or PyTorch fallback.  Loading
fails loudly when the shared object is missing (build it with
``python -m logkv_b200.build``) and every call's return code is checked.
"""
from __future__ import annotations

import ctypes
import os

import torch

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "liblogkv_b200.so")

ERRORS = {-1: "shape out of the supported range", -2: "unsupported storage dtype",
          -3: "workspace missing or too small", -4: "null or misaligned pointer",
          -5: "shape needs more shared memory than one SM has",
          -6: "the cache state lives on another device than the current one"}

DTYPE_CODES = {torch.float32: 0, torch.bfloat16: 1}

FLUSH_STAGES = ("snapshot", "span_cut", "score_attach", "choose", "seed_plan", "prepare", "cascade",
                "pool_rewrite", "window_shift")
COUNTERS = ("storage_read", "stage_read", "survivor", "fill", "clear", "carry", "gather", "flushes", "exact_cuts",
            "ties", "seq_lanes")
TIE_KINDS = {1: "attach_cost", 2: "direct", 3: "nearest", 4: "seed_pick", 5: "seed_nearest", 6: "beta_cut",
             7: "alpha_order", 8: "alpha_swap", 9: "ward_min", 10: "ward_budget"}


ROUTE_ATTACH, ROUTE_UNIFIED = 0, 1   # logkv_layout_t.route (LOGKV_ROUTE_*)
# Per-lane words of the unified route (logkv_read_unified).
UNIFIED_WORDS = ("cand_live", "cand_active", "cand_merges", "cand_rounds", "glob_live", "glob_active", "glob_merges",
                 "glob_rounds", "glob_rows", "old_clusters", "candidates", "cand_exact_form", "glob_exact_form",
                 "ward_merges", "unused14", "unused15")


class Layout(ctypes.Structure):
    _fields_ = [("batch", ctypes.c_int32), ("groups", ctypes.c_int32), ("dim", ctypes.c_int32),
                ("clusters", ctypes.c_int32), ("levels", ctypes.c_int32), ("slots", ctypes.c_int32),
                ("recent_capacity", ctypes.c_int32), ("exact", ctypes.c_int32), ("span_cap", ctypes.c_int32),
                ("beta", ctypes.c_int32), ("dtype", ctypes.c_int32), ("eta", ctypes.c_float),
                ("g0", ctypes.c_float), ("lam", ctypes.c_float), ("route", ctypes.c_int32),
                ("merge_passes", ctypes.c_int32)]


STATE_FIELDS = ["level_k", "level_v", "level_w", "level_p_lo", "level_p_hi", "level_sum_wp", "level_order",
                "pad_mask", "level_count", "centroid", "n_eff", "n_total", "p_hi_c", "level0_phase", "alive",
                "s_h", "recent_k", "recent_k_raw", "recent_v", "recent_pos", "recent_ends", "alpha_k_raw",
                "alpha_v", "alpha_pos", "alpha_valid", "alpha_span_len", "alpha_span_closed", "alpha_nspans",
                "alpha_rowcount", "alpha_count"]


class State(ctypes.Structure):
    _fields_ = [(name, ctypes.c_void_p) for name in STATE_FIELDS]


class Tie(ctypes.Structure):
    _fields_ = [(name, ctypes.c_int32) for name in ("kind", "flush", "batch", "group", "cluster", "index", "first",
                                                     "second")] + [("gap", ctypes.c_float), ("value", ctypes.c_float)]


class Plan(ctypes.Structure):
    _fields_ = [("idx", ctypes.c_void_p), ("anchor", ctypes.c_void_p), ("valid", ctypes.c_void_p),
                ("width", ctypes.c_void_p), ("width_max", ctypes.c_void_p), ("vslot", ctypes.c_void_p),
                ("vanchor", ctypes.c_void_p), ("nvalid", ctypes.c_void_p), ("exact_rows", ctypes.c_void_p),
                ("nexact", ctypes.c_void_p)]


class Rope(ctypes.Structure):
    _fields_ = [("cos", ctypes.c_void_p), ("sin", ctypes.c_void_p), ("rows", ctypes.c_int32),
                ("rope_n", ctypes.c_int32), ("dtype", ctypes.c_int32)]


class Prefix(ctypes.Structure):
    _fields_ = [("k", ctypes.c_void_p), ("v", ctypes.c_void_p), ("mass", ctypes.c_void_p),
                ("length", ctypes.c_void_p), ("capacity", ctypes.c_int32)]


class Chunk(ctypes.Structure):
    """logkv_chunk_t: a chunk of window rows (include/logkv_b200.h)."""
    _fields_ = [("k", ctypes.c_void_p), ("k_strides", ctypes.c_int64 * 3), ("k_raw", ctypes.c_void_p),
                ("k_raw_strides", ctypes.c_int64 * 3), ("v", ctypes.c_void_p), ("v_strides", ctypes.c_int64 * 3),
                ("positions", ctypes.c_void_p), ("pos_strides", ctypes.c_int64 * 2), ("pos0", ctypes.c_int64),
                ("ends", ctypes.c_void_p), ("n", ctypes.c_int32)]


class AttentionArgs(ctypes.Structure):
    _fields_ = [("q", ctypes.c_void_p), ("k_new", ctypes.c_void_p), ("v_new", ctypes.c_void_p),
                ("out", ctypes.c_void_p), ("heads", ctypes.c_int32), ("tokens", ctypes.c_int32),
                ("q_offset", ctypes.c_int32), ("q_tokens", ctypes.c_int32), ("recent_count", ctypes.c_int32),
                ("causal", ctypes.c_int32), ("scale", ctypes.c_float), ("qx", ctypes.c_float),
                ("q_stride", ctypes.c_int32)]


_lib = None


def lib() -> ctypes.CDLL:
    """Load the library once; raise if it was not built."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise RuntimeError(f"logkv_b200 CUDA library missing at {LIB_PATH}; run `python -m logkv_b200.build`")
        handle = ctypes.CDLL(LIB_PATH)
        handle.logkv_flush_workspace_bytes.restype = ctypes.c_size_t
        handle.logkv_flush_workspace_bytes.argtypes = [ctypes.POINTER(Layout), ctypes.c_int32]
        handle.logkv_flush.restype = ctypes.c_int
        handle.logkv_flush.argtypes = [ctypes.POINTER(Layout), ctypes.POINTER(State), ctypes.c_int32,
                                       ctypes.c_int32, ctypes.c_void_p, ctypes.c_size_t, ctypes.c_void_p]
        handle.logkv_stream_capture_id.restype = ctypes.c_int
        handle.logkv_stream_capture_id.argtypes = [ctypes.c_void_p, ctypes.POINTER(ctypes.c_ulonglong)]
        handle.logkv_read_status.restype = ctypes.c_int
        handle.logkv_read_status.argtypes = [ctypes.c_void_p, ctypes.POINTER(ctypes.c_int32), ctypes.c_void_p]
        handle.logkv_flush_profiled.restype = ctypes.c_int
        handle.logkv_flush_profiled.argtypes = [ctypes.POINTER(Layout), ctypes.POINTER(State), ctypes.c_int32,
                                                ctypes.c_int32, ctypes.c_void_p, ctypes.c_size_t, ctypes.c_void_p,
                                                ctypes.POINTER(ctypes.c_void_p), ctypes.c_int32]
        handle.logkv_read_counters.restype = ctypes.c_int
        handle.logkv_read_counters.argtypes = [ctypes.c_void_p, ctypes.POINTER(ctypes.c_uint64), ctypes.c_int32,
                                               ctypes.c_void_p]
        handle.logkv_read_unified.restype = ctypes.c_int
        handle.logkv_read_unified.argtypes = [ctypes.POINTER(Layout), ctypes.c_int32, ctypes.c_void_p,
                                              ctypes.POINTER(ctypes.c_int32), ctypes.c_int32, ctypes.c_void_p]
        P = ctypes.POINTER
        I64 = P(ctypes.c_int64)
        handle.logkv_window_append.restype = ctypes.c_int
        handle.logkv_window_append.argtypes = [P(Layout), P(State), ctypes.c_void_p, I64, ctypes.c_void_p, I64,
                                               ctypes.c_void_p, I64, ctypes.c_void_p, I64, ctypes.c_int64,
                                               ctypes.c_void_p, ctypes.c_int32, ctypes.c_int32, ctypes.c_void_p]
        handle.logkv_flush_chunk.restype = ctypes.c_int
        handle.logkv_flush_chunk.argtypes = [P(Layout), P(State), ctypes.c_int32, ctypes.c_int32, P(Chunk),
                                             ctypes.c_void_p, ctypes.c_size_t, ctypes.c_void_p]
        handle.logkv_flush_chunk_profiled.restype = ctypes.c_int
        handle.logkv_flush_chunk_profiled.argtypes = [P(Layout), P(State), ctypes.c_int32, ctypes.c_int32, P(Chunk),
                                                      ctypes.c_void_p, ctypes.c_size_t, ctypes.c_void_p,
                                                      ctypes.POINTER(ctypes.c_void_p), ctypes.c_int32]
        handle.logkv_read_ties.restype = ctypes.c_int
        handle.logkv_read_ties.argtypes = [ctypes.c_void_p, P(Tie), ctypes.c_int32, P(ctypes.c_int64), ctypes.c_int32,
                                           ctypes.c_void_p]
        flush_args = [P(Layout), P(State), ctypes.c_int32, ctypes.c_int32, ctypes.c_void_p, ctypes.c_size_t]
        handle.logkv_flush_scores.restype = ctypes.c_int
        handle.logkv_flush_scores.argtypes = flush_args + [ctypes.c_void_p]
        handle.logkv_flush_commit.restype = ctypes.c_int
        handle.logkv_flush_commit.argtypes = flush_args + [ctypes.c_void_p, ctypes.c_int32, ctypes.c_void_p]
        handle.logkv_flush_commit_strided.restype = ctypes.c_int
        handle.logkv_flush_commit_strided.argtypes = flush_args + [ctypes.c_void_p, ctypes.c_int32, ctypes.c_int64,
                                                                   ctypes.c_void_p]
        for name in ("logkv_flush_decide", "logkv_flush_apply"):
            getattr(handle, name).restype = ctypes.c_int
            getattr(handle, name).argtypes = flush_args + [ctypes.c_void_p]
        handle.logkv_flush_partials.restype = ctypes.c_int
        handle.logkv_flush_partials.argtypes = [P(Layout), ctypes.c_int32, ctypes.c_void_p,
                                                P(P(ctypes.c_float)), P(ctypes.c_size_t)]
        handle.logkv_flush_oplog_append.restype = ctypes.c_int
        handle.logkv_flush_oplog_append.argtypes = [P(Layout), ctypes.c_int32, ctypes.c_void_p, ctypes.c_void_p,
                                                    ctypes.c_void_p, ctypes.c_int32, ctypes.c_void_p]
        handle.logkv_tape_bytes.restype = ctypes.c_size_t
        handle.logkv_tape_bytes.argtypes = [P(Layout), ctypes.c_int32]
        handle.logkv_flush_record.restype = ctypes.c_int
        handle.logkv_flush_record.argtypes = flush_args + [ctypes.c_void_p, ctypes.c_size_t, ctypes.c_void_p]
        handle.logkv_flush_commit_record.restype = ctypes.c_int
        handle.logkv_flush_commit_record.argtypes = flush_args[:6] + [ctypes.c_void_p, ctypes.c_int32, ctypes.c_int64,
                                                                      ctypes.c_void_p, ctypes.c_size_t,
                                                                      ctypes.c_void_p]
        handle.logkv_flush_replay.restype = ctypes.c_int
        handle.logkv_flush_replay.argtypes = flush_args + [ctypes.c_void_p, ctypes.c_size_t, ctypes.c_void_p]
        handle.logkv_attention_plan.restype = ctypes.c_int
        handle.logkv_attention_plan.argtypes = [P(Layout), P(State), P(Plan), ctypes.c_void_p]
        handle.logkv_pack_prefix.restype = ctypes.c_int
        handle.logkv_pack_prefix.argtypes = [P(Layout), P(State), P(Plan), P(Rope), P(Prefix), ctypes.c_void_p,
                                             ctypes.c_void_p]
        handle.logkv_pack_mid.restype = ctypes.c_int
        handle.logkv_pack_mid.argtypes = [P(Layout), P(State), P(Plan), P(Rope), ctypes.c_int32, ctypes.c_int32,
                                          ctypes.c_int32, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int32,
                                          ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int32, ctypes.c_int32,
                                          ctypes.c_int32, ctypes.c_void_p, ctypes.c_void_p]
        handle.logkv_attention_workspace_bytes.restype = ctypes.c_size_t
        handle.logkv_attention_workspace_bytes.argtypes = [P(Layout), ctypes.c_int32, ctypes.c_int32, ctypes.c_int32]
        handle.logkv_attention.restype = ctypes.c_int
        handle.logkv_attention.argtypes = [P(Layout), P(State), P(Prefix), P(AttentionArgs), ctypes.c_void_p,
                                           ctypes.c_size_t, ctypes.c_void_p]
        _lib = handle
    return _lib


def check(code: int, what: str) -> None:
    if code != 0:
        reason = ERRORS.get(code, f"CUDA error {code}")
        raise RuntimeError(f"{what} failed: {reason}")


def capture_id(device: torch.device) -> int:
    """Id of the CUDA-graph capture the current stream of `device` takes part in, 0 if none."""
    out = ctypes.c_ulonglong(0)
    check(lib().logkv_stream_capture_id(ctypes.c_void_p(stream_ptr(device)), ctypes.byref(out)),
          "logkv_stream_capture_id")
    return int(out.value)


def stream_ptr(device: torch.device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def ptr(t: torch.Tensor) -> int:
    if not t.is_cuda:
        raise ValueError("logkv_b200 kernels need CUDA tensors")
    if not t.is_contiguous():
        raise ValueError("logkv_b200 kernels need contiguous tensors")
    return t.data_ptr()
