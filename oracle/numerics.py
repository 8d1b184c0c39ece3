"""Bit-level bf16/fp16 <-> fp32 conversions for the oracle (test infrastructure only).

bf16 values are carried as their uint16 bit patterns; fp16 values as
numpy.float16.  Rounding is round-to-nearest-even, the rounding torch uses for
``tensor.to(torch.bfloat16)`` and the GPU's ``cvt.rn``.
"""
from __future__ import annotations

import numpy as np


def bf16_bits_to_f32(bits: np.ndarray) -> np.ndarray:
    """bf16 bit patterns (uint16) -> float32 (exact)."""
    return (bits.astype(np.uint32) << np.uint32(16)).view(np.float32)


def f32_to_bf16_bits(x: np.ndarray) -> np.ndarray:
    """float32 -> bf16 bit patterns with round-to-nearest-even; NaN stays NaN."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    u = x.view(np.uint32)
    nan = (u & np.uint32(0x7FFFFFFF)) > np.uint32(0x7F800000)
    lsb = (u >> np.uint32(16)) & np.uint32(1)
    rounded = (u + np.uint32(0x7FFF) + lsb) >> np.uint32(16)
    out = rounded.astype(np.uint16)
    out[nan] = ((u[nan] >> np.uint32(16)) | np.uint32(0x0040)).astype(np.uint16)
    return out


def to_f32(arr: np.ndarray, dtype: str) -> np.ndarray:
    """Storage array (uint16 bf16 bits or float16) -> float32 values."""
    if dtype == "bf16":
        return bf16_bits_to_f32(arr)
    if dtype == "f16":
        return arr.astype(np.float32)
    raise ValueError(dtype)


def from_f32(x: np.ndarray, dtype: str) -> np.ndarray:
    """float32 values -> storage array of ``dtype`` (round to nearest even)."""
    if dtype == "bf16":
        return f32_to_bf16_bits(x)
    if dtype == "f16":
        return np.asarray(x, dtype=np.float32).astype(np.float16)
    raise ValueError(dtype)
