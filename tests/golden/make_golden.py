"""Generates the golden fixtures in this directory from the reference's own code.

Run where a checkout of the reference is available, with MOE_REFERENCE_SRC
naming its ``src`` directory:

    MOE_REFERENCE_SRC=<checkout>/src python tests/golden/make_golden.py

It imports ``src/triton_grouped_gemm.py`` of Hongyu15/moe-overlap and records,
on the CPU:
  * ``expert_offsets_from_recv_counts`` (:300-323) on lists and tensors of
    several dtypes, including int32 wrap-around;
  * ``_build_work_queue`` (:240-297) for ragged offsets and several tile shapes;
  * ``reference_grouped_gemm`` (:446-457) on small ragged fp16/bf16 problems
    (inputs stored) and on the BASELINE config-1 problem (inputs regenerated
    from the seed by tests/_inputs.py; a row subset and per-row sums stored).

The fixtures are what the oracle is pinned against (tests/test_oracle_golden.py);
nothing that runs on the GPU box reads the reference.
"""
from __future__ import annotations

import os
import sys
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent
REPO = HERE.parents[1]
sys.path.insert(0, str(REPO))
sys.dont_write_bytecode = True

from tests._inputs import gemm_inputs, to_storage  # noqa: E402

REF_SRC = Path(os.environ["MOE_REFERENCE_SRC"]) if "MOE_REFERENCE_SRC" in os.environ else None


def _import_reference():
    if REF_SRC is None:
        raise SystemExit("set MOE_REFERENCE_SRC to the reference checkout's src directory")
    sys.path.insert(0, str(REF_SRC))
    import triton_grouped_gemm as tg  # noqa: PLC0415

    return tg


def offsets_cases(tg) -> dict:
    cases = {
        "list_small": ([3, 0, 5, 7], None),
        "list_empty": ([], None),
        "t_int32": (torch.tensor([128] * 8, dtype=torch.int32), None),
        "t_int64_wrap": (torch.tensor([2**31 + 5, 1, -7, 2**33 + 3], dtype=torch.int64), None),
        "t_float": (torch.tensor([1.9, 2.2, -0.5, 3.0], dtype=torch.float32), None),
        "t_2d": (torch.tensor([[4, 5], [6, 7]], dtype=torch.int32), None),
        "t_int32_out_int64": (torch.tensor([100, 200, 0, 50], dtype=torch.int32), torch.int64),
        "t_int64_out_int64": (torch.tensor([2**31, 2**31, 1], dtype=torch.int64), torch.int64),
    }
    out = {}
    for name, (counts, dtype) in cases.items():
        kwargs = {} if dtype is None else {"dtype": dtype}
        res = tg.expert_offsets_from_recv_counts(counts, **kwargs)
        src = counts if isinstance(counts, list) else counts.numpy()
        out[f"offsets/{name}/counts"] = np.asarray(src)
        out[f"offsets/{name}/dtype"] = np.array(str(res.dtype))
        out[f"offsets/{name}/result"] = res.numpy()
    return out


def work_queue_cases(tg) -> dict:
    offsets_list = {
        "ragged": [0, 3, 3, 73, 202, 203, 459, 459, 759, 1783],
        "uniform": [0, 512, 1024, 1536, 2048],
        "nonmono": [0, 100, 50, 150],
        "allzero": [0, 0, 0],
    }
    out = {}
    for oname, offs in offsets_list.items():
        for n, bm, bn in ((1000, 128, 128), (4096, 128, 256), (96, 64, 32)):
            we, wm, wn = tg._build_work_queue(torch.tensor(offs, dtype=torch.int32), n, bm, bn)
            key = f"wq/{oname}/{n}_{bm}_{bn}"
            out[key + "/offsets"] = np.asarray(offs, dtype=np.int32)
            out[key + "/expert"] = we.numpy()
            out[key + "/tile_m"] = wm.numpy()
            out[key + "/tile_n"] = wn.numpy()
    return out


SMALL_GEMMS = [
    # name, counts, k, n, dtype, seed
    ("ragged_f16", [3, 0, 17, 40], 32, 24, "f16", 11),
    ("ragged_bf16", [1, 9, 0, 30, 2], 48, 40, "bf16", 12),
    ("single_bf16", [33], 64, 16, "bf16", 13),
]


def gemm_cases(tg) -> dict:
    out = {}
    for name, counts, k, n, dtype, seed in SMALL_GEMMS:
        a, b, off = gemm_inputs(counts, k, n, dtype, seed)
        c = tg.reference_grouped_gemm(a, b, off)
        rows = int(off[-1])
        out[f"gemm/{name}/a"] = to_storage(a)
        out[f"gemm/{name}/b"] = to_storage(b)
        out[f"gemm/{name}/offsets"] = off.numpy()
        out[f"gemm/{name}/c"] = to_storage(c[:rows])
        out[f"gemm/{name}/dtype"] = np.array(dtype)
    # E=8, 128 rows each, H=512, F=1024, fp16, seed 0.
    a, b, off = gemm_inputs([128] * 8, 512, 1024, "f16", seed=0)
    c = tg.reference_grouped_gemm(a, b, off)
    rows = np.arange(0, 1024, 16)
    out["gemm/cfg1/rows"] = rows
    out["gemm/cfg1/c_rows"] = to_storage(c[rows])
    out["gemm/cfg1/row_sums"] = c.double().sum(dim=1).numpy()
    out["gemm/cfg1/a_sum"] = np.array(a.double().sum().item())
    out["gemm/cfg1/b_sum"] = np.array(b.double().sum().item())
    return out


def main() -> None:
    tg = _import_reference()
    data = {}
    data.update(offsets_cases(tg))
    data.update(work_queue_cases(tg))
    data.update(gemm_cases(tg))
    path = HERE / "grouped_gemm_golden.npz"
    np.savez_compressed(path, **data)
    print(f"wrote {path} ({path.stat().st_size} bytes, {len(data)} arrays)")


if __name__ == "__main__":
    main()
