"""Round fp32 arrays to bf16 / fp16 precision (kept in fp32), numpy only.

Test infrastructure for the oracle (see oracle/__init__.py).
"""
from __future__ import annotations

import numpy as np


def round_to_bf16(x: np.ndarray) -> np.ndarray:
    """fp32 -> nearest bf16 (ties to even), returned as fp32 values.

    bf16 keeps the top 16 bits of the fp32 encoding; rounding adds half an
    ulp of the kept part plus the tie-breaking bit before truncating.  NaN
    payloads are preserved as quiet NaNs.
    """
    x = np.ascontiguousarray(x, dtype=np.float32)
    bits = x.view(np.uint32).astype(np.uint64)
    lsb = (bits >> 16) & 1
    rounded = ((bits + 0x7FFF + lsb) >> 16) << 16
    out = rounded.astype(np.uint32).view(np.float32).copy()
    nan = np.isnan(x)
    out[nan] = np.float32("nan")
    return out


def round_to_fp16(x: np.ndarray) -> np.ndarray:
    """fp32 -> nearest fp16 (ties to even, numpy's IEEE cast), returned as fp32 values."""
    with np.errstate(over="ignore"):
        return np.asarray(x, dtype=np.float32).astype(np.float16).astype(np.float32)


def round_to(x: np.ndarray, dtype: str) -> np.ndarray:
    if dtype == "bf16":
        return round_to_bf16(x)
    if dtype == "fp16":
        return round_to_fp16(x)
    if dtype == "fp32":
        return np.asarray(x, dtype=np.float32)
    raise ValueError(f"unknown dtype {dtype!r}")
