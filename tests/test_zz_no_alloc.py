"""GPU check of moe_grouped_gemm_noalloc, the allocation-free grouped GEMM entry point.

That entry point serves callers that cannot allocate device memory (code under
a host framework whose memory pool owns the GPU, latency-critical loops where
an allocation could stall the device): its atomic tile-queue counter lives in a
fixed device array inside the library instead of a caller-provided buffer.

The test calls it through the C ABI twice in a row, and checks both results
against the regular moe_grouped_gemm entry point and against the CPU oracle's
fp32-accumulated per-expert loop, with the tolerance the other GEMM tests use.  The second call only passes if the shared counter was cleared
again, since the first call leaves it at (tiles + grid).  This file sorts last
so a run that stops at the first failure has already run every other test; it
passes alone in a fresh process as well.
"""
import ctypes

import numpy as np
import pytest
import torch

from moe_overlap_b200 import _lib
from oracle import grouped_gemm as og
from oracle.numerics import to_f32
from tests._inputs import gemm_inputs, to_storage, zipf_counts

pytestmark = pytest.mark.gpu


def _within_gemm_tolerance(got: torch.Tensor, want, rows: int) -> None:
    """bf16 rule of the GEMM tests: max_abs <= 2^-7 max|ref| + 1e-2, rel-L2 <= 1e-2.
    ``want`` is a device tensor or the oracle's bf16 storage array."""
    g = to_f32(to_storage(got[:rows]), "bf16").astype(np.float64)
    w_store = to_storage(want[:rows]) if isinstance(want, torch.Tensor) else want[:rows]
    w = to_f32(w_store, "bf16").astype(np.float64)
    diff = np.abs(g - w)
    atol = 2.0 ** -7 * float(np.abs(w).max()) + 1e-2
    rel_l2 = float(np.linalg.norm(diff) / max(np.linalg.norm(w), 1e-30))
    assert float(diff.max()) <= atol and rel_l2 <= 1e-2, (float(diff.max()), rel_l2)


def test_noalloc_entry_point_matches_regular_entry_point(cuda_device):
    lib = _lib.load()
    counts = zipf_counts(2500, 12, 1.2, seed=21)
    a_cpu, b_cpu, off_cpu = gemm_inputs(counts, 384, 520, "bf16", seed=22)
    oracle_c, _ = og.grouped_gemm(to_storage(a_cpu), to_storage(b_cpu), off_cpu.numpy(), "bf16")
    a, b, off = a_cpu.to(cuda_device), b_cpu.to(cuda_device), off_cpu.to(cuda_device)
    m_total, k = a.shape
    num_experts, _, n = b.shape
    stream = torch.cuda.current_stream(cuda_device).cuda_stream
    status = torch.zeros(1, dtype=torch.int32, device=cuda_device)

    # Regular entry point: caller-provided counter.
    want = torch.empty((m_total, n), dtype=a.dtype, device=cuda_device)
    counter = torch.zeros(1, dtype=torch.int32, device=cuda_device)
    rc = lib.moe_grouped_gemm(
        a.data_ptr(), a.stride(0), b.data_ptr(), b.stride(0), b.stride(1), b.stride(2),
        want.data_ptr(), want.stride(0), off.data_ptr(), 0, m_total, k, n, num_experts,
        _lib.MOE_DTYPE_BF16, _lib.MOE_ACT_NONE, 7, 1, counter.data_ptr(), status.data_ptr(),
        stream)
    assert rc == _lib.MOE_OK, _lib.status_string(rc)

    rows = int(off[-1])
    for _ in range(2):
        got = torch.full((m_total, n), float("nan"), dtype=a.dtype, device=cuda_device)
        rc = lib.moe_grouped_gemm_noalloc(
            a.data_ptr(), a.stride(0), b.data_ptr(), b.stride(0), b.stride(1), b.stride(2),
            got.data_ptr(), got.stride(0), off.data_ptr(), 0, m_total, k, n, num_experts,
            _lib.MOE_DTYPE_BF16, _lib.MOE_ACT_NONE, 7, ctypes.c_void_p(status.data_ptr()),
            stream)
        assert rc == _lib.MOE_OK, _lib.status_string(rc)
        torch.cuda.synchronize(cuda_device)
        assert int(status.item()) == 0, _lib.status_string(int(status.item()))
        assert not torch.isnan(got[:rows]).any()
        _within_gemm_tolerance(got, want, rows)
        _within_gemm_tolerance(got, oracle_c, rows)


def test_noalloc_entry_point_refuses_oversized_problems(cuda_device):
    lib = _lib.load()
    rc = lib.moe_grouped_gemm_noalloc(16, 2048, 16, 2048 * 1024, 1024, 1, 16, 1024 * 1024 * 64, 16,
                                      0, 1 << 30, 2048, 1024 * 1024 * 64, 16,
                                      _lib.MOE_DTYPE_BF16, _lib.MOE_ACT_NONE, 148, None, None)
    assert rc == _lib.MOE_ERR_CAPACITY
