"""The reference's CPU grouped GEMM, restated in torch -- TEST INFRASTRUCTURE ONLY.

``reference_grouped_gemm`` (src/triton_grouped_gemm.py:446-457) is the
reference's own CPU path for the grouped GEMM: a Python loop over the experts
that multiplies each expert's row segment by its weight matrix with one torch
matmul in the input dtype (bf16 or fp16; the CPU backend accumulates in fp32
and rounds once), writing into a ``torch.empty`` output.  This module restates
that loop so that ``bench.py`` can time it on the GPU box's host cores (the
reference's sources cannot travel there): it is the timed reference arm and the
``cpu_baseline`` leg, never the product path.
"""
from __future__ import annotations

import torch


def grouped_gemm_loop(a: torch.Tensor, b: torch.Tensor, offsets, experts=None,
                      out: torch.Tensor | None = None) -> torch.Tensor:
    """``out[off[e]:off[e+1]] = a[off[e]:off[e+1]] @ b[e]`` for each expert with rows.

    ``a`` [M, K] and ``b`` [E, K, N] are CPU tensors of one dtype; ``offsets`` is
    a sequence of E+1 ints.  ``experts`` restricts the loop to those expert ids
    (a bounded sample of the same work); ``out`` is reused when given.
    """
    off = [int(v) for v in offsets]
    if out is None:
        out = torch.empty((a.shape[0], b.shape[2]), dtype=a.dtype)
    for e in (range(b.shape[0]) if experts is None else experts):
        s, t = off[e], off[e + 1]
        if t > s:
            torch.matmul(a[s:t], b[e], out=out[s:t])
    return out


def loop_flops(a_shape, b_shape, offsets, experts=None) -> int:
    """2*rows*K*N summed over the experts the loop multiplies (real rows only)."""
    off = [int(v) for v in offsets]
    k, n = int(b_shape[1]), int(b_shape[2])
    ids = range(int(b_shape[0])) if experts is None else experts
    return sum(2 * max(0, off[e + 1] - off[e]) * k * n for e in ids)
