"""Generates ``fp8_golden.npz`` from the reference's own FP8 helpers.

Run where a checkout of the reference is available, with MOE_REFERENCE_SRC
naming its ``src`` directory (DeepEP is vendored beside it):

    MOE_REFERENCE_SRC=<checkout>/src python tests/golden/make_golden_fp8.py

It imports ``thirdParty/DeepEP/tests/utils.py`` and records, on the CPU, for
seeded bf16 inputs (normal rows, rows of mixed magnitude, an all-zero group and
values at the e4m3 rounding ties):
  * ``per_token_cast_to_fp8`` (:50-58): the e4m3 bytes and float32 scales that
    DeepEP's FP8 dispatch carries (buffer.py:338-342);
  * ``per_token_cast_back`` (:61-75): the bf16 rows rebuilt from them.
tests/test_oracle_fp8.py pins oracle/fp8.py to these arrays; nothing that runs
on the GPU box reads the reference.
"""
from __future__ import annotations

import os
import sys
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent
REPO = HERE.parents[1]
sys.dont_write_bytecode = True


def make_inputs() -> np.ndarray:
    """bf16 bits [24, 512]: seeded rows, including the edge cases named above."""
    g = torch.Generator().manual_seed(2024)
    x = torch.randn(24, 512, generator=g)
    x[1] *= 1e-3                       # small magnitudes (subnormal e4m3 codes after scaling)
    x[2] *= 300.0                      # large magnitudes
    x[3, :128] = 0.0                   # an all-zero group: amax clamps to 1e-4
    x[4, 128:256] = torch.linspace(-2.0, 2.0, 128)
    x[5] = torch.where(torch.arange(512) % 2 == 0, x[5], -x[5] * 1e-5)  # mixed magnitudes
    return x.to(torch.bfloat16).view(torch.int16).numpy().view(np.uint16)


def main() -> None:
    src = os.environ.get("MOE_REFERENCE_SRC")
    if not src:
        raise SystemExit("set MOE_REFERENCE_SRC to the reference checkout's src directory")
    sys.path.insert(0, str(Path(src).resolve().parent / "thirdParty" / "DeepEP" / "tests"))
    import utils as deep_ep_test_utils  # thirdParty/DeepEP/tests/utils.py

    bits = make_inputs()
    x = torch.from_numpy(bits.view(np.int16)).view(torch.bfloat16)
    q, scales = deep_ep_test_utils.per_token_cast_to_fp8(x)
    back = deep_ep_test_utils.per_token_cast_back(q, scales)
    np.savez_compressed(
        HERE / "fp8_golden.npz",
        x=bits,
        q=q.view(torch.uint8).numpy(),
        scales=scales.numpy().astype(np.float32),
        back=back.view(torch.int16).numpy().view(np.uint16),
    )
    print(f"wrote {HERE / 'fp8_golden.npz'}: x {bits.shape}, scales {tuple(scales.shape)}")


if __name__ == "__main__":
    main()
