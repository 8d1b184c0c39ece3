"""Oracle for the FP8 dispatch payload (test infrastructure only).

DeepEP's dispatch accepts, instead of bf16 rows, a pair (x_fp8 [T, H]
float8_e4m3fn, x_scales [T, H/128] float32) and moves both unchanged
(thirdParty/DeepEP/deep_ep/buffer.py:338-342; the per-128 scales are copied
next to each row, csrc/kernels/intranode.cu:397-402).  The pair is made and
undone as DeepEP's tests do:
  * ``quantize_per128``   follows ``per_token_cast_to_fp8``
    (thirdParty/DeepEP/tests/utils.py:50-58): per row and 128-column group,
    amax = max|x| clamped to 1e-4, q = e4m3(x * ((1 / amax) * 448)), scale = amax / 448
    (torch evaluates the ``448.0 / amax`` written there as a reciprocal times 448);
  * ``dequantize_per128`` follows ``per_token_cast_back`` (:61-75):
    bf16(float(q) * scale).
The e4m3 conversion is restated from the format (1 sign, 4 exponent bits with
bias 7, 3 mantissa bits, no infinities; the largest finite value is 448):
round to nearest, ties to even, and values past 448 clamp to 448.  Every step
is a float32 operation, so the result is bit-exact.
"""
from __future__ import annotations

import numpy as np

from .numerics import bf16_bits_to_f32, f32_to_bf16_bits

E4M3_MAX = 448.0
GROUP = 128


def e4m3_encode(v) -> np.ndarray:
    """float32 values -> e4m3 bytes (uint8), round-to-nearest-even, clamped to +-448."""
    f = np.asarray(v, dtype=np.float32).astype(np.float64)
    sign = np.signbit(f)
    a = np.minimum(np.abs(f), E4M3_MAX)
    code = np.zeros(a.shape, dtype=np.int64)
    normal = a >= 2.0 ** -6
    # normal numbers: 8 * 2^e <= m * 2^(e-3) with m in [8, 16)
    e = np.floor(np.log2(np.where(normal, a, 1.0))).astype(np.int64)
    m = np.rint(a / np.exp2(e - 3)).astype(np.int64)  # ties to even; may reach 16
    carry = m == 16
    e = np.where(carry, e + 1, e)
    m = np.where(carry, 8, m)
    code_n = ((e + 7) << 3) | (m - 8)
    # subnormals: multiples of 2^-9 below 2^-6 (rounding up to 8 gives the smallest normal)
    q = np.rint(a / 2.0 ** -9).astype(np.int64)
    code = np.where(normal, code_n, q)
    code = np.minimum(code, 0x7E)  # 448
    return (code | (sign.astype(np.int64) << 7)).astype(np.uint8)


def e4m3_decode(b) -> np.ndarray:
    """e4m3 bytes -> float32 (0x7F/0xFF, the format's NaN, decode as NaN)."""
    b = np.asarray(b, dtype=np.uint8).astype(np.int64)
    sign = np.where(b & 0x80, -1.0, 1.0)
    e = (b >> 3) & 0xF
    m = b & 0x7
    val = np.where(e == 0, m * 2.0 ** -9, (8 + m) * np.exp2(e - 10.0))
    val = np.where((b & 0x7F) == 0x7F, np.nan, val)
    return (sign * val).astype(np.float32)


def quantize_per128(x_bits: np.ndarray) -> tuple[np.ndarray, np.ndarray]:
    """bf16 bits [T, H] (H a multiple of 128) -> (e4m3 bytes [T, H], float32 scales [T, H/128])."""
    x = bf16_bits_to_f32(np.asarray(x_bits, dtype=np.uint16))
    t, h = x.shape
    g = x.reshape(t, h // GROUP, GROUP)
    amax = np.maximum(np.abs(g).max(axis=2), np.float32(1e-4)).astype(np.float32)
    # ``448.0 / x_amax`` with a tensor on the right is evaluated by torch as
    # ``x_amax.reciprocal() * 448.0``: two float32 roundings, not one division.
    mult = ((np.float32(1.0) / amax).astype(np.float32) * np.float32(E4M3_MAX)).astype(np.float32)
    prod = (g * mult[:, :, None]).astype(np.float32)
    q = e4m3_encode(prod).reshape(t, h)
    scales = (amax / np.float32(E4M3_MAX)).astype(np.float32)
    return q, scales


def dequantize_per128(q: np.ndarray, scales: np.ndarray) -> np.ndarray:
    """(e4m3 bytes [T, H], float32 scales [T, H/128]) -> bf16 bits [T, H]."""
    qf = e4m3_decode(q)
    t, h = qf.shape
    prod = (qf.reshape(t, h // GROUP, GROUP) * np.asarray(scales, np.float32)[:, :, None]).astype(np.float32)
    return f32_to_bf16_bits(prod.reshape(t, h))
