"""Rounding helpers for the oracle: emulate bf16 / f16 storage in numpy float32.

numpy has no bfloat16; a bf16 value is carried as the float32 with the same
value.  ``round_bf16`` rounds float32 to the nearest bf16 (ties to even), the
conversion torch's ``.to(torch.bfloat16)`` performs.
"""
from __future__ import annotations

import numpy as np


def round_bf16(x) -> np.ndarray:
    x = np.ascontiguousarray(np.asarray(x, dtype=np.float32))
    bits = x.view(np.uint32)
    nan = np.isnan(x)
    lsb = (bits >> np.uint32(16)) & np.uint32(1)
    rounded = (bits + np.uint32(0x7FFF) + lsb) & np.uint32(0xFFFF0000)
    out = rounded.view(np.float32).copy()
    out[nan] = np.nan
    return out


def round_f16(x) -> np.ndarray:
    return np.asarray(x, dtype=np.float32).astype(np.float16).astype(np.float32)


def round_to(x, dtype: str) -> np.ndarray:
    if dtype == "bfloat16":
        return round_bf16(x)
    if dtype == "float16":
        return round_f16(x)
    if dtype == "float32":
        return np.asarray(x, dtype=np.float32)
    raise ValueError(dtype)


def ulp_distance_bf16(a, b) -> np.ndarray:
    """Distance in bf16 units-in-the-last-place between two arrays of bf16 values."""
    def ordered(v):
        i = (np.asarray(v, dtype=np.float32).view(np.int32) >> 16).astype(np.int64)
        return np.where(i < 0, -(i & 0x7FFF), i)
    return np.abs(ordered(a) - ordered(b))
