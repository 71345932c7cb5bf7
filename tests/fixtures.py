"""Helpers to load the reference-generated golden stream fixtures."""
from __future__ import annotations

import json
import os
import sys

import numpy as np

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")
sys.path.insert(0, GOLDEN)
from streams import CONFIGS, make_stream  # noqa: E402

from oracle.numerics import bf16_bits_to_f32  # noqa: E402

FLOAT_FIELDS = {"level_k", "level_v", "recent_k", "recent_k_raw", "recent_v", "alpha_k_raw", "alpha_v"}


def config(name: str) -> dict:
    return next(c for c in CONFIGS if c["name"] == name)


def load(name: str):
    with open(os.path.join(GOLDEN, "index.json")) as fh:
        index = json.load(fh)
    z = np.load(os.path.join(GOLDEN, index[name]))
    steps: dict = {}
    for key in z.files:
        step, field = key.split("/", 1)
        steps.setdefault(int(step[4:]), {})[field] = z[key]
    return [steps[i] for i in sorted(steps)]


def as_values(arr: np.ndarray, field: str) -> np.ndarray:
    """Fixture array -> comparable numpy values (bf16 bit patterns widened to float32)."""
    if arr.dtype == np.uint16:
        return bf16_bits_to_f32(arr)
    return arr
