"""Pins the CPU oracle to golden vectors produced by the reference's own code.

The fixtures (tests/golden/grouped_gemm_golden.npz) come from
tests/golden/make_golden.py, which imports src/triton_grouped_gemm.py of the
reference.  Integer results must match bit for bit; GEMM outputs (torch CPU
matmul in the reference vs numpy fp32 here, both accumulated in fp32 with a
different summation order and rounded once) may differ by at most two units in
the last place, and only on a small fraction of the elements.
"""
from pathlib import Path

import numpy as np
import pytest
import torch

from oracle import grouped_gemm as og
from oracle.numerics import bf16_bits_to_f32, f32_to_bf16_bits, to_f32
from tests._inputs import gemm_inputs, to_storage

GOLDEN = np.load(Path(__file__).parent / "golden" / "grouped_gemm_golden.npz")


def _names(prefix: str) -> list[str]:
    return sorted({k.split("/")[1] for k in GOLDEN.files if k.startswith(prefix + "/")})


@pytest.mark.parametrize("name", _names("offsets"))
def test_oracle_offsets_match_reference(name):
    counts = GOLDEN[f"offsets/{name}/counts"]
    want = GOLDEN[f"offsets/{name}/result"]
    got = og.expert_offsets_from_recv_counts(counts.reshape(-1)).astype(want.dtype)
    assert got.dtype == want.dtype and np.array_equal(got, want)


@pytest.mark.parametrize("name", _names("offsets"))
def test_library_host_offsets_match_reference(name):
    """The product's host routine (CPU tensors / lists) against the reference."""
    import moe_overlap_b200 as mo

    counts = GOLDEN[f"offsets/{name}/counts"]
    want = GOLDEN[f"offsets/{name}/result"]
    dtype = getattr(torch, str(GOLDEN[f"offsets/{name}/dtype"]).split(".")[-1])
    arg = counts.tolist() if name.startswith("list") else torch.from_numpy(counts)
    got = mo.expert_offsets_from_recv_counts(arg, dtype=dtype)
    assert got.dtype == dtype and got.device.type == "cpu"
    assert np.array_equal(got.numpy(), want)


@pytest.mark.parametrize("key", sorted({k.rsplit("/", 1)[0] for k in GOLDEN.files if k.startswith("wq/")}))
def test_oracle_work_queue_matches_reference(key):
    n, bm, bn = (int(v) for v in key.split("/")[-1].split("_"))
    we, wm, wn = og.build_work_queue(GOLDEN[key + "/offsets"], n, bm, bn)
    assert np.array_equal(we, GOLDEN[key + "/expert"])
    assert np.array_equal(wm, GOLDEN[key + "/tile_m"])
    assert np.array_equal(wn, GOLDEN[key + "/tile_n"])


def _ulp_diff_fraction(got_f32: np.ndarray, want_f32: np.ndarray, mant: int) -> tuple[float, float]:
    diff = np.abs(got_f32.astype(np.float64) - want_f32.astype(np.float64))
    ulp = np.exp2(np.floor(np.log2(np.maximum(np.abs(want_f32), 2.0 ** -14))) - mant)
    return float(np.mean(diff > ulp * 1.0001)), float(np.max(diff / ulp)) if diff.size else 0.0


@pytest.mark.parametrize("name", _names("gemm"))
def test_oracle_gemm_matches_reference(name):
    if name == "cfg1":
        a, b, off = gemm_inputs([128] * 8, 512, 1024, "f16", seed=0)
        assert a.double().sum().item() == float(GOLDEN["gemm/cfg1/a_sum"])
        assert b.double().sum().item() == float(GOLDEN["gemm/cfg1/b_sum"])
        c, defined = og.grouped_gemm(to_storage(a), to_storage(b), off.numpy(), "f16")
        rows = GOLDEN["gemm/cfg1/rows"]
        got = to_f32(c[rows], "f16")
        want = to_f32(GOLDEN["gemm/cfg1/c_rows"], "f16")
        frac, worst = _ulp_diff_fraction(got, want, 10)
        assert worst <= 2.0 + 1e-6 and frac <= 1e-3, (frac, worst)
        sums = to_f32(c, "f16").astype(np.float64).sum(axis=1)
        np.testing.assert_allclose(sums, GOLDEN["gemm/cfg1/row_sums"], rtol=0, atol=0.05)
        return
    dtype = str(GOLDEN[f"gemm/{name}/dtype"])
    a, b = GOLDEN[f"gemm/{name}/a"], GOLDEN[f"gemm/{name}/b"]
    off = GOLDEN[f"gemm/{name}/offsets"]
    c, defined = og.grouped_gemm(a, b, off, dtype)
    rows = int(off[-1])
    assert defined[:rows].all()
    got, want = to_f32(c[:rows], dtype), to_f32(GOLDEN[f"gemm/{name}/c"], dtype)
    frac, worst = _ulp_diff_fraction(got, want, 7 if dtype == "bf16" else 10)
    assert worst <= 2.0 + 1e-6 and frac <= 1e-2, (frac, worst)


def test_bf16_rounding_matches_torch():
    g = torch.Generator().manual_seed(0)
    x = torch.randn(1 << 16, generator=g) * torch.logspace(-30, 30, 1 << 16)
    x[:4] = torch.tensor([float("inf"), float("-inf"), float("nan"), 0.0])
    want = x.to(torch.bfloat16).view(torch.int16).numpy().view(np.uint16)
    got = f32_to_bf16_bits(x.numpy())
    same = (got == want) | (np.isnan(bf16_bits_to_f32(got)) & np.isnan(bf16_bits_to_f32(want)))
    assert same.all()


def test_oracle_empty_experts_give_zero_output():
    a, b, off = gemm_inputs([0, 0], 16, 8, "bf16", seed=0, m_extra=5)
    c, defined = og.grouped_gemm(to_storage(a), to_storage(b), off.numpy(), "bf16")
    assert defined.all() and not c.any()
