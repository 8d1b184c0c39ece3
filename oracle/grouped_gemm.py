"""Oracle for the grouped-GEMM path (test infrastructure only).

Restates, in numpy, the reference's
  * ``expert_offsets_from_recv_counts``  src/triton_grouped_gemm.py:300-323
  * ``_build_work_queue``               src/triton_grouped_gemm.py:240-297
  * ``reference_grouped_gemm``          src/triton_grouped_gemm.py:446-457, with
    the fp32-accumulate-then-round contract of ``_gemm_tile`` (:80-95)
and the exact GELU the layer applies after the up-projection
(src/train_moe_baseline.py:243, ``F.gelu`` default = erf form).
"""
from __future__ import annotations

import numpy as np
from scipy.special import erf

from .numerics import from_f32, to_f32


def expert_offsets_from_recv_counts(counts) -> np.ndarray:
    """int64 ``[0, cumsum(counts)]``; counts are narrowed to int32 first.

    Follows src/triton_grouped_gemm.py:315-323: ``t.to(torch.int32)``, then an
    integer cumsum (which torch promotes to int64) concatenated after a zero.
    The caller casts the int64 result to the requested dtype (``.to(dtype)``,
    :323), e.g. with ``.astype(np.int32)`` which wraps like torch's cast.
    """
    c = np.asarray(counts)
    if c.dtype.kind == "f":
        c = np.trunc(c)
    c32 = c.astype(np.int64).astype(np.int32) if c.size else np.zeros(0, np.int32)
    out = np.zeros(c32.size + 1, dtype=np.int64)
    np.cumsum(c32.astype(np.int64), out=out[1:])
    return out


def build_work_queue(offsets, n_size: int, block_m: int, block_n: int):
    """(work_expert, work_tile_m, work_tile_n) int32 lists.

    Follows src/triton_grouped_gemm.py:253-292: counts = clamp(off[e+1]-off[e], 0),
    ceil(count/block_m) row tiles times ceil(n/block_n) column tiles per expert,
    listed expert-major, then tile_m, with tile_n fastest.
    """
    off = np.asarray(offsets, dtype=np.int64)
    counts = np.maximum(off[1:] - off[:-1], 0)
    tiles_m = (counts + block_m - 1) // block_m
    tiles_n = (n_size + block_n - 1) // block_n
    we, wm, wn = [], [], []
    for e, tm in enumerate(tiles_m.tolist()):
        if tm <= 0 or tiles_n <= 0:
            continue
        m_idx, n_idx = np.meshgrid(np.arange(tm), np.arange(tiles_n), indexing="ij")
        we.append(np.full(tm * tiles_n, e, dtype=np.int32))
        wm.append(m_idx.reshape(-1).astype(np.int32))
        wn.append(n_idx.reshape(-1).astype(np.int32))
    if not we:
        z = np.zeros(0, dtype=np.int32)
        return z, z.copy(), z.copy()
    return np.concatenate(we), np.concatenate(wm), np.concatenate(wn)


def gelu_erf(x: np.ndarray) -> np.ndarray:
    """Exact GELU 0.5*x*(1+erf(x/sqrt(2))) evaluated in float64."""
    x64 = np.asarray(x, dtype=np.float64)
    return 0.5 * x64 * (1.0 + erf(x64 / np.sqrt(2.0)))


def grouped_gemm_f32(a: np.ndarray, b: np.ndarray, offsets, dtype: str,
                     activation: str | None = None) -> tuple[np.ndarray, np.ndarray]:
    """fp32 result of the grouped GEMM before rounding, and the defined-row mask.

    ``a``: [M, K] storage array, ``b``: [E, K, N] storage array (uint16 bf16
    bits or float16).  For each expert with off[e+1] > off[e] the rows
    off[e]:off[e+1] are ``a[rows] @ b[e]`` accumulated in fp32 (the per-expert
    loop of src/triton_grouped_gemm.py:450-456); other rows are undefined in
    the reference (``torch.empty``) and are returned as zero with mask False.
    """
    off = np.asarray(offsets, dtype=np.int64)
    m_total = a.shape[0]
    n_size = b.shape[2]
    af = to_f32(a, dtype)
    out = np.zeros((m_total, n_size), dtype=np.float32)
    defined = np.zeros(m_total, dtype=bool)
    for e in range(b.shape[0]):
        s, t = int(off[e]), int(off[e + 1])
        if t <= s:
            continue
        acc = af[s:t] @ to_f32(b[e], dtype)
        if activation == "gelu":
            acc = gelu_erf(acc).astype(np.float32)
        out[s:t] = acc
        defined[s:t] = True
    return out, defined


def grouped_gemm(a: np.ndarray, b: np.ndarray, offsets, dtype: str,
                 activation: str | None = None) -> tuple[np.ndarray, np.ndarray]:
    """Rounded grouped-GEMM output (storage dtype) and the defined-row mask.

    When no expert has rows the whole output is zero and every row is defined
    (src/triton_grouped_gemm.py:369-371).
    """
    acc, defined = grouped_gemm_f32(a, b, offsets, dtype, activation)
    if not defined.any():
        defined[:] = True
    return from_f32(acc, dtype), defined


def gelu_erf_grad(x: np.ndarray) -> np.ndarray:
    """d/dx of exact GELU: Phi(x) + x * phi(x), in float64."""
    x64 = np.asarray(x, dtype=np.float64)
    return 0.5 * (1.0 + erf(x64 / np.sqrt(2.0))) + x64 * np.exp(-0.5 * x64 * x64) / np.sqrt(2.0 * np.pi)


def grouped_gemm_ex(a, b, offsets, dtype: str, activation=None, row_scale=None, aux_in=None):
    """Extended epilogue: v = acc * row_scale; returns (C, aux_out) as storage arrays
    and the defined-row mask.  aux_out = v, except gelu'(v) for "gelu_save_grad".
    activation None / "gelu" / "gelu_save_grad" (GELU(v)) / "dgelu" (v * gelu'(aux_in))
    / "mul_aux" (v * aux_in)."""
    acc, defined = grouped_gemm_f32(a, b, offsets, dtype)
    if row_scale is not None:
        acc = (acc * np.asarray(row_scale, np.float32)[:, None]).astype(np.float32)
    aux = from_f32(acc, dtype)
    if activation == "gelu":
        out = gelu_erf(acc).astype(np.float32)
    elif activation == "gelu_save_grad":
        out = gelu_erf(acc).astype(np.float32)
        aux = from_f32(gelu_erf_grad(acc).astype(np.float32), dtype)
    elif activation == "dgelu":
        out = (acc * gelu_erf_grad(to_f32(aux_in, dtype))).astype(np.float32)
    elif activation == "mul_aux":
        out = (acc * to_f32(aux_in, dtype)).astype(np.float32)
    else:
        out = acc
    return from_f32(out, dtype), aux, defined


def wgrad(a, b, offsets, dtype: str):
    """C[e] = A[off[e]:off[e+1]]^T @ B[off[e]:off[e+1]] in fp32, rounded; [E, M, N]."""
    off = np.asarray(offsets, dtype=np.int64)
    af, bf = to_f32(a, dtype), to_f32(b, dtype)
    out = np.zeros((len(off) - 1, af.shape[1], bf.shape[1]), dtype=np.float32)
    for e in range(len(off) - 1):
        s, t = int(off[e]), int(off[e + 1])
        if t > s:
            out[e] = af[s:t].T @ bf[s:t]
    return from_f32(out, dtype)
