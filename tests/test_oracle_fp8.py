"""The FP8 payload oracle (oracle/fp8.py) against the reference's own FP8 helpers.

``fp8_golden.npz`` holds DeepEP's ``per_token_cast_to_fp8`` / ``per_token_cast_back``
(thirdParty/DeepEP/tests/utils.py:50-75) run on seeded bf16 rows
(tests/golden/make_golden_fp8.py).  The oracle must reproduce the e4m3 bytes, the
scales and the rebuilt bf16 rows bit for bit; its e4m3 rounding is also checked
against torch's float8_e4m3fn conversion on every code, every rounding tie and
random values.
"""
from pathlib import Path

import numpy as np
import torch

from oracle import fp8

GOLDEN = Path(__file__).resolve().parent / "golden" / "fp8_golden.npz"


def test_quantize_matches_deepep_per_token_cast_to_fp8():
    g = np.load(GOLDEN)
    q, scales = fp8.quantize_per128(g["x"])
    assert np.array_equal(q, g["q"])
    assert np.array_equal(scales.view(np.uint32), g["scales"].view(np.uint32))


def test_dequantize_matches_deepep_per_token_cast_back():
    g = np.load(GOLDEN)
    assert np.array_equal(fp8.dequantize_per128(g["q"], g["scales"]), g["back"])


def test_e4m3_rounding_matches_torch_on_codes_ties_and_random_values():
    codes = torch.arange(256, dtype=torch.uint8).view(torch.float8_e4m3fn).float().numpy()
    grid = np.unique(codes[np.isfinite(codes)]).astype(np.float32)
    mids = ((grid[1:].astype(np.float64) + grid[:-1]) / 2).astype(np.float32)
    rng = np.random.default_rng(5)
    vals = np.concatenate([grid, mids, np.nextafter(mids, np.float32(np.inf)),
                           np.nextafter(mids, np.float32(-np.inf)),
                           (rng.standard_normal(50000) * 100).astype(np.float32),
                           (rng.standard_normal(50000) * 0.01).astype(np.float32)])
    vals = vals[np.abs(vals) <= 448.0]
    want = torch.from_numpy(vals).to(torch.float8_e4m3fn).view(torch.uint8).numpy()
    assert np.array_equal(fp8.e4m3_encode(vals), want)
    dec = fp8.e4m3_decode(np.arange(256, dtype=np.uint8))
    finite = np.isfinite(codes)
    assert np.array_equal(dec[finite], codes[finite]) and np.isnan(dec[~finite]).all()


def test_values_past_the_largest_code_clamp_to_448():
    assert fp8.e4m3_encode(np.array([500.0, -1e6, 464.0], np.float32)).tolist() == [0x7E, 0xFE, 0x7E]
