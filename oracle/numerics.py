"""Float helpers for the oracle (test infrastructure only).

bfloat16 values are carried as float32 arrays holding exactly representable
bf16 values; ``round_bf16`` is IEEE round-to-nearest-even on the float32 bits,
which is what a ``tensor.to(torch.bfloat16)`` cast does on CPU and what
``__float2bfloat16_rn`` does on the GPU.
"""
from __future__ import annotations

import numpy as np

F32 = np.float32


def round_bf16(x: np.ndarray) -> np.ndarray:
    """Round float32 values to the nearest bfloat16 (ties to even); NaN stays NaN."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    bits = x.view(np.uint32).astype(np.uint64)
    lsb = (bits >> 16) & 1
    rounded = ((bits + 0x7FFF + lsb) >> 16) << 16
    nan = np.isnan(x)
    out = (rounded & 0xFFFFFFFF).astype(np.uint32).view(np.float32)
    return np.where(nan, x, out).astype(np.float32)


def to_storage(x: np.ndarray, dtype: str) -> np.ndarray:
    """Cast float32 values to the cache storage dtype ('fp32' or 'bf16'), kept as float32."""
    x = np.asarray(x, dtype=np.float32)
    return round_bf16(x) if dtype == "bf16" else x.copy()


def bf16_bits_to_f32(bits: np.ndarray) -> np.ndarray:
    """uint16 bf16 bit patterns -> float32 values."""
    return (np.asarray(bits, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


def f32_to_bf16_bits(x: np.ndarray) -> np.ndarray:
    """float32 values (already bf16-exact or not) -> rounded uint16 bf16 bit patterns."""
    return (round_bf16(x).view(np.uint32) >> 16).astype(np.uint16)


def dsum(x: np.ndarray) -> np.ndarray:
    """Canonical feature-axis reduction: left-to-right float32 sum over the last axis from +0.0.

    The reference reduces feature vectors with torch's vectorised CPU order,
    which depends on the host's SIMD width; its decisions are compared with
    this order only through the argmin/threshold they feed.  The CUDA kernels
    use exactly this order (one thread walks the features), so CUDA and oracle
    agree bit for bit on every distance, energy and cost.
    """
    x = np.asarray(x, dtype=np.float32)
    if x.shape[-1] == 0:
        return np.zeros(x.shape[:-1], dtype=np.float32)
    # ufunc.accumulate is evaluated strictly left to right in float32; +0.0 added
    # first changes nothing but the sign of an all-negative-zero sum.
    return (np.add.accumulate(x, axis=-1, dtype=np.float32)[..., -1] + np.float32(0.0)).astype(np.float32)


def ddot(a: np.ndarray, b: np.ndarray) -> np.ndarray:
    """Canonical dot product over the last axis: products rounded to float32, summed by ``dsum``."""
    return dsum((np.asarray(a, np.float32) * np.asarray(b, np.float32)).astype(np.float32))


def seq_sum(rows: np.ndarray) -> np.ndarray:
    """Left-to-right float32 sum over axis 0 starting from +0.0.

    Matches ``torch.segment_reduce(..., 'sum')`` and reductions over a short
    non-innermost axis on CPU, both of which accumulate in index order.
    """
    rows = np.asarray(rows, dtype=np.float32)
    if rows.shape[0] == 0:
        return np.zeros(rows.shape[1:], dtype=np.float32)
    return (np.float32(0.0) + np.add.accumulate(rows, axis=0, dtype=np.float32)[-1]).astype(np.float32)
