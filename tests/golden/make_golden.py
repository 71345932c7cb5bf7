"""Generate golden fixtures by running the UNMODIFIED reference (HourunLi/LogKV) on CPU.

Test infrastructure only. This script imports the reference's own modules
(`litgpt.log_kv_cache`, `alpha_log_kv`, `beta_log_kv`, `log_kv_position`) from a
read-only checkout whose path is given by ``--reference`` (or the
``LOGKV_REFERENCE`` environment variable), drives the reference cache through a
seeded streaming workload and records, after every ``add_recent`` call, every
``named_buffers()`` entry plus the host mirrors the reference treats as
authoritative.  At every third step it also records, for the chunk about to be committed,
the reference's CPU slot-attention output (``log_kv_chunk_attention``, math
path) over the whole chunk and over its first two tokens (the decode shape),
the mid-anchor attention plan (``_semantic_attention_plan``) and the torch
packer's output (``log_kv_pack.pack_mid_kv(..., backend="torch")``).

The reference's ``litgpt/__init__`` imports ``lightning``, which is not needed
by the cache modules; a stub import hook stands in for it (test scaffolding,
nothing of the reference is modified or copied).

Usage:  python tests/golden/make_golden.py --reference <checkout> [--out tests/golden]
"""
from __future__ import annotations

import argparse
import importlib.abc
import importlib.machinery
import json
import os
import sys
import types

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, HERE)
from streams import CONFIGS, UNIFIED_CONFIGS, make_stream  # noqa: E402


def install_shim(reference: str) -> None:
    class _Stub(types.ModuleType):
        def __getattr__(self, name):
            if name.startswith("__"):
                raise AttributeError(name)
            return type(name, (), {"__init__": lambda self, *a, **k: None,
                                   "__bool__": lambda self: False,
                                   "__call__": lambda self, *a, **k: None})

    class _Finder(importlib.abc.MetaPathFinder, importlib.abc.Loader):
        def find_spec(self, name, path, target=None):
            if name.split(".")[0] in ("lightning", "lightning_utilities"):
                return importlib.machinery.ModuleSpec(name, self, is_package=True)
            return None

        def create_module(self, spec):
            mod = _Stub(spec.name)
            mod.__path__ = []
            return mod

        def exec_module(self, module):
            pass

    sys.meta_path.insert(0, _Finder())
    pkg = types.ModuleType("litgpt")
    pkg.__path__ = [os.path.join(reference, "litgpt")]
    sys.modules["litgpt"] = pkg


MIRRORS = ("_semantic_counts", "_semantic_alive", "_semantic_p_hi_c", "_semantic_n_total",
           "_semantic_level0_phase", "_semantic_current_segment")


def to_np(t: torch.Tensor) -> np.ndarray:
    t = t.detach().cpu()
    if t.dtype == torch.bfloat16:
        return t.view(torch.int16).numpy().view(np.uint16).copy()
    return t.numpy().copy()


def record_state(cache, out: dict, prefix: str) -> None:
    for name, buf in cache.named_buffers():
        if buf is None or name in ("cos_cache", "sin_cache"):
            continue
        out[f"{prefix}/{name}"] = to_np(buf)
    for name in MIRRORS:
        out[f"{prefix}/{name}"] = np.asarray(getattr(cache, name), dtype=np.int64)
    spans = cache._alpha_spans
    n = max((len(r) for r in spans), default=0)
    table = np.zeros((len(spans), max(n, 1), 2), dtype=np.int64)
    nspan = np.zeros(len(spans), dtype=np.int64)
    for b, row in enumerate(spans):
        nspan[b] = len(row)
        for i, (length, closed) in enumerate(row):
            table[b, i] = (length, int(closed))
    out[f"{prefix}/alpha_spans"] = table
    out[f"{prefix}/alpha_nspans"] = nspan
    width = max((len(r) for r in cache._alpha_positions), default=0)
    pos = np.full((len(spans), max(width, 1)), -1, dtype=np.int64)
    for b, row in enumerate(cache._alpha_positions):
        pos[b, :len(row)] = row
    out[f"{prefix}/alpha_positions"] = pos
    out[f"{prefix}/scalars"] = np.asarray([cache.alpha_count, cache.recent_count, cache.token_count,
                                           cache.B_prime, cache.L_alloc], dtype=np.int64)


def run_config(cfg: dict, outdir: str) -> str:
    from litgpt.log_kv_cache import LogStructuredKVCache, log_kv_chunk_attention
    from litgpt.log_kv_pack import pack_mid_kv

    torch.set_num_threads(4)
    stream = make_stream(cfg)
    dtype = torch.float32 if cfg["dtype"] == "fp32" else torch.bfloat16
    cos = torch.from_numpy(stream["cos"])
    sin = torch.from_numpy(stream["sin"])
    if cfg.get("rope_dtype", "fp32") == "bf16":
        cos, sin = cos.to(torch.bfloat16), sin.to(torch.bfloat16)
    cache = LogStructuredKVCache(
        (cfg["batch"], cfg["groups"], cfg["max_seq"], cfg["dim"]),
        (cfg["batch"], cfg["groups"], cfg["max_seq"], cfg["dim"]),
        B=cfg["slots"], recent_size=cfg["recent"], dtype=dtype,
        semantic_clusters=True, cluster_k_max=cfg["clusters"], semantic_anchor_mode="mid",
        semantic_flush_granularity=cfg["granularity"], semantic_centroid_backend="sequential",
        semantic_replay_updates=True, allocate_second_order=False,
        alpha_exact_tokens=cfg["exact"], alpha_span_max_tokens=cfg["span_cap"],
        beta_novelty=cfg["beta"], beta_adaptive_merge=cfg["beta"],
        semantic_s_h=cfg.get("s_h"), cos_cache=cos, sin_cache=sin, rope_n_elem=cfg["dim"],
        semantic_unified_route=cfg.get("unified", False), semantic_merge_passes=cfg.get("merge_passes", 1),
    )
    out: dict = {}
    for step, chunk in enumerate(stream["chunks"]):
        k = torch.from_numpy(chunk["k"]).to(dtype)
        kr = torch.from_numpy(chunk["k_raw"]).to(dtype)
        v = torch.from_numpy(chunk["v"]).to(dtype)
        q = torch.from_numpy(chunk["q"]).to(dtype)
        pos = torch.from_numpy(chunk["pos"]) if chunk.get("pos") is not None else None
        if chunk.get("attend"):
            scale = cfg["dim"] ** -0.5
            pack_dim = ((cfg["dim"] + 1 + 7) // 8) * 8
            with torch.no_grad():
                att = log_kv_chunk_attention(cache, q, k, v, scale, 0.0)
                dec = log_kv_chunk_attention(cache, q[:, :, :2], k[:, :, :2], v[:, :, :2], scale, 0.0)
                plan = cache._semantic_attention_plan()
                ka, va = pack_mid_kv(cache, plan, k, v, pack_dim, backend="torch")
            out[f"step{step}/attention"] = to_np(att.float())
            out[f"step{step}/decode_attention"] = to_np(dec.float())
            out[f"step{step}/plan_idx"] = to_np(plan[0])
            out[f"step{step}/plan_anchor"] = to_np(plan[1])
            out[f"step{step}/plan_valid"] = to_np(plan[3])
            out[f"step{step}/pack_k"] = to_np(ka)
            out[f"step{step}/pack_v"] = to_np(va)
        cache.add_recent(k, v, k_raw=kr, input_pos=pos, span_ends=chunk["span_ends"].tolist())
        record_state(cache, out, f"step{step}")
    path = os.path.join(outdir, f"stream_{cfg['name']}.npz")
    np.savez_compressed(path, **out)
    return path


def main() -> None:
    parser = argparse.ArgumentParser()
    parser.add_argument("--reference", default=os.environ.get("LOGKV_REFERENCE"))
    parser.add_argument("--out", default=HERE)
    parser.add_argument("--only", default=None)
    args = parser.parse_args()
    if not args.reference:
        raise SystemExit("pass --reference <reference checkout> or set LOGKV_REFERENCE")
    install_shim(args.reference)
    index = {}
    index_path = os.path.join(args.out, "index.json")
    if os.path.exists(index_path):
        with open(index_path) as fh:
            index = json.load(fh)
    for cfg in CONFIGS + UNIFIED_CONFIGS:
        if args.only and cfg["name"] != args.only:
            continue
        path = run_config(cfg, args.out)
        index[cfg["name"]] = os.path.basename(path)
        print("wrote", path, os.path.getsize(path))
    with open(index_path, "w") as fh:
        json.dump(index, fh, indent=1, sort_keys=True)


if __name__ == "__main__":
    main()
