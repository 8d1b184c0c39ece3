"""Seeded input builders shared by the tests, the smoke check and the bench.

Inputs are drawn on the CPU with a torch.Generator so the oracle and the GPU
see identical bits; they are moved to the device afterwards.
"""
from __future__ import annotations

import numpy as np
import torch

TORCH_DTYPE = {"bf16": torch.bfloat16, "f16": torch.float16}


def to_storage(t: torch.Tensor) -> np.ndarray:
    """CPU bf16/fp16 tensor -> numpy storage (uint16 bf16 bits or float16)."""
    t = t.detach().cpu().contiguous()
    if t.dtype == torch.bfloat16:
        return t.view(torch.int16).numpy().view(np.uint16)
    if t.dtype == torch.float16:
        return t.numpy()
    raise TypeError(t.dtype)


def gemm_inputs(counts, k: int, n: int, dtype: str, seed: int, w_std: float = 0.02,
                m_extra: int = 0):
    """A ~ N(0,1) [sum(counts)+m_extra, k], B ~ N(0, w_std) [E, k, n], int32 offsets."""
    g = torch.Generator().manual_seed(seed)
    td = TORCH_DTYPE[dtype]
    m = int(sum(counts)) + m_extra
    a = torch.randn(m, k, generator=g).to(td)
    b = (torch.randn(len(counts), k, n, generator=g) * w_std).to(td)
    offsets = torch.zeros(len(counts) + 1, dtype=torch.int32)
    if len(counts):
        offsets[1:] = torch.cumsum(torch.tensor(counts, dtype=torch.int64), 0).to(torch.int32)
    return a, b, offsets


def zipf_counts(total: int, num_experts: int, s: float, seed: int, zero_least: bool = True):
    """Multinomial counts from Zipf(s) popularity over a seeded expert permutation.

    The least popular expert's probability is set to zero so that at least one
    expert receives no rows (a plain Zipf(1.2) draw over 16 experts never does).
    """
    g = torch.Generator().manual_seed(seed)
    ranks = torch.arange(1, num_experts + 1, dtype=torch.float64)
    p = ranks.pow(-s)
    if zero_least:
        p[-1] = 0.0
    p = p / p.sum()
    perm = torch.randperm(num_experts, generator=g)
    probs = torch.empty_like(p)
    probs[perm] = p
    draws = torch.multinomial(probs, total, replacement=True, generator=g)
    return torch.bincount(draws, minlength=num_experts).tolist()
