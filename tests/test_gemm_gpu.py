"""GPU parity of the grouped GEMM (C-ABI path) against the CPU oracle.

Tolerances (written here, from the path's stated bf16/fp16 contract):
  bf16: max_abs <= 2^-7 * max|ref| + 1e-2 and rel_L2 <= 1e-2
  fp16: max_abs <= 2^-10 * max|ref| + 1e-3 and rel_L2 <= 2e-3
and, since both sides accumulate in fp32 and round once, at most 0.1% of the
elements may differ from the oracle by more than one unit in the last place.
"""
import zlib

import numpy as np
import pytest
import torch

import moe_overlap_b200 as mo
from moe_overlap_b200 import _lib
from oracle import grouped_gemm as og
from oracle.numerics import to_f32
from tests._inputs import gemm_inputs, to_storage, zipf_counts

pytestmark = pytest.mark.gpu


def _ulp(x: np.ndarray, dtype: str) -> np.ndarray:
    mant = 7 if dtype == "bf16" else 10
    ax = np.maximum(np.abs(x), np.float32(2.0 ** -14))
    return np.exp2(np.floor(np.log2(ax)) - mant)


def assert_matches_oracle(out: torch.Tensor, ref: np.ndarray, defined: np.ndarray, dtype: str):
    o = to_f32(to_storage(out), dtype)[defined]
    r = to_f32(ref, dtype)[defined]
    if r.size == 0:
        return
    diff = np.abs(o.astype(np.float64) - r.astype(np.float64))
    max_abs = float(diff.max())
    rel_l2 = float(np.linalg.norm(diff) / max(np.linalg.norm(r.astype(np.float64)), 1e-30))
    ref_max = float(np.abs(r).max())
    if dtype == "bf16":
        atol, rtol = 2.0 ** -7 * ref_max + 1e-2, 1e-2
    else:
        atol, rtol = 2.0 ** -10 * ref_max + 1e-3, 2e-3
    beyond_ulp = float(np.mean(diff > _ulp(r, dtype) * 1.0001))
    msg = f"max_abs={max_abs:.3e} (tol {atol:.3e}) rel_l2={rel_l2:.3e} (tol {rtol}) >1ulp={beyond_ulp:.2e}"
    assert max_abs <= atol and rel_l2 <= rtol, msg
    assert beyond_ulp <= 1e-3, msg


CASES = [
    # name, counts, k, n, dtype, num_sms, atomic
    ("cfg1_f16", [128] * 8, 512, 1024, "f16", 148, False),
    ("ragged_bf16_atomic", [3, 0, 70, 129, 1, 256, 0, 300], 64, 96, "bf16", 148, True),
    ("k_tail_striped_7sms", [5, 200, 17], 72, 40, "bf16", 7, False),
    ("few_sms_atomic_f16", [130, 1, 260], 136, 520, "f16", 3, True),
    ("one_expert_bf16", [1000], 256, 264, "bf16", 148, True),
    ("k_pad_70", [10, 20, 0, 33], 70, 24, "bf16", 148, False),
    ("n_pad_30", [10, 20], 64, 30, "f16", 148, True),
    # last tiles on both sides of every swap boundary: N = rows rounded up to 16 from
    # 1 to 224 rows (64-row A box up to 128 rows, the full box above), full tiles above
    ("swap_boundaries", [16, 17, 112, 113, 127, 128, 129, 143, 144, 145, 200, 223, 224, 225,
                         240, 255, 256, 257, 481], 128, 264, "bf16", 148, True),
]


@pytest.mark.parametrize("name,counts,k,n,dtype,num_sms,atomic", CASES, ids=[c[0] for c in CASES])
def test_grouped_gemm_matches_oracle(cuda_device, name, counts, k, n, dtype, num_sms, atomic):
    a, b, off = gemm_inputs(counts, k, n, dtype, seed=zlib.crc32(name.encode()) % 1000)
    c = mo.persistent_grouped_gemm(
        a.to(cuda_device), b.to(cuda_device), off.to(cuda_device), num_sms=num_sms,
        use_atomic_queue=atomic,
    )
    mo.check_status(cuda_device, sync=True)
    ref, defined = og.grouped_gemm(to_storage(a), to_storage(b), off.numpy(), dtype)
    assert c.shape == (a.shape[0], n) and c.dtype == a.dtype and c.is_contiguous()
    assert_matches_oracle(c, ref, defined, dtype)


def test_atomic_and_striped_are_bitwise_equal(cuda_device):
    counts = zipf_counts(3000, 16, 1.2, seed=3)
    a, b, off = gemm_inputs(counts, 256, 512, "bf16", seed=4)
    a, b, off = a.to(cuda_device), b.to(cuda_device), off.to(cuda_device)
    c1 = mo.persistent_grouped_gemm(a, b, off, num_sms=148, use_atomic_queue=False)
    c2 = mo.persistent_grouped_gemm(a, b, off, num_sms=148, use_atomic_queue=True)
    c3 = mo.persistent_grouped_gemm(a, b, off, num_sms=5, use_atomic_queue=True)
    mo.check_status(cuda_device, sync=True)
    rows = int(off[-1])
    assert torch.equal(c1[:rows], c2[:rows]) and torch.equal(c1[:rows], c3[:rows])


def test_all_experts_empty_gives_zeros(cuda_device):
    a, b, off = gemm_inputs([0, 0, 0], 64, 64, "bf16", seed=1, m_extra=50)
    c = mo.persistent_grouped_gemm(a.to(cuda_device), b.to(cuda_device), off.to(cuda_device))
    mo.check_status(cuda_device, sync=True)
    assert c.shape == (50, 64) and torch.count_nonzero(c).item() == 0


def test_rows_past_last_offset_untouched_and_int64_offsets(cuda_device):
    a, b, off = gemm_inputs([7, 0, 140], 128, 256, "bf16", seed=2, m_extra=33)
    out = torch.full((a.shape[0], 256), 3.0, dtype=torch.bfloat16, device=cuda_device)
    mo.grouped_gemm(a.to(cuda_device), b.to(cuda_device), off.to(torch.int64).to(cuda_device),
                    out=out)
    mo.check_status(cuda_device, sync=True)
    ref, defined = og.grouped_gemm(to_storage(a), to_storage(b), off.numpy(), "bf16")
    assert_matches_oracle(out, ref, defined, "bf16")
    assert bool((out[147:] == 3.0).all())


def test_fused_gelu_matches_oracle(cuda_device):
    counts = [100, 0, 257, 31, 150, 224, 473]
    a, b, off = gemm_inputs(counts, 512, 384, "bf16", seed=5, w_std=0.05)
    c = mo.grouped_gemm(a.to(cuda_device), b.to(cuda_device), off.to(cuda_device),
                        activation="gelu")
    mo.check_status(cuda_device, sync=True)
    ref, defined = og.grouped_gemm(to_storage(a), to_storage(b), off.numpy(), "bf16",
                                   activation="gelu")
    assert_matches_oracle(c, ref, defined, "bf16")


def test_k_major_weight_view(cuda_device):
    counts = [64, 200, 0, 129]
    a, b, off = gemm_inputs(counts, 192, 320, "bf16", seed=6)
    b_t = b.transpose(1, 2).contiguous().to(cuda_device)  # [E, N, K] storage
    b_view = b_t.transpose(1, 2)  # [E, K, N] view with unit K stride
    assert b_view.stride(1) == 1
    c = mo.persistent_grouped_gemm(a.to(cuda_device), b_view, off.to(cuda_device), num_sms=148)
    mo.check_status(cuda_device, sync=True)
    ref, defined = og.grouped_gemm(to_storage(a), to_storage(b), off.numpy(), "bf16")
    assert_matches_oracle(c, ref, defined, "bf16")


@pytest.mark.parametrize("cfg", ["cfg2", "cfg3"])
def test_baseline_configs_full_size(cuda_device, cfg):
    if cfg == "cfg2":
        counts, atomic = [512] * 16, False
    else:
        counts, atomic = zipf_counts(16384, 16, 1.2, seed=0), True
        assert min(counts) == 0 and max(counts) > 0.25 * 16384
    a, b, off = gemm_inputs(counts, 2048, 4096, "bf16", seed=0)
    c = mo.persistent_grouped_gemm(a.to(cuda_device), b.to(cuda_device), off.to(cuda_device),
                                   num_sms=148, use_atomic_queue=atomic)
    mo.check_status(cuda_device, sync=True)
    ref, defined = og.grouped_gemm(to_storage(a), to_storage(b), off.numpy(), "bf16")
    assert_matches_oracle(c, ref, defined, "bf16")


@pytest.mark.parametrize("block_m,block_n", [(128, 128), (64, 32), (128, 256)])
def test_tile_list_matches_reference_work_queue(cuda_device, block_m, block_n):
    counts = [3, 0, 70, 129, 1, 256, 0, 300, 1024]
    off = torch.tensor(og.expert_offsets_from_recv_counts(counts).astype(np.int32))
    n = 1000
    we, wm, wn = mo.tile_list(off.to(cuda_device), int(off[-1]), n, block_m, block_n, order=0)
    re, rm, rn = og.build_work_queue(off.numpy(), n, block_m, block_n)
    assert np.array_equal(we.cpu().numpy(), re)
    assert np.array_equal(wm.cpu().numpy(), rm)
    assert np.array_equal(wn.cpu().numpy(), rn)
    # The kernel's own order is a permutation of the same tiles.
    ke, km, kn = mo.tile_list(off.to(cuda_device), int(off[-1]), n, block_m, block_n, order=1)
    got = sorted(zip(ke.tolist(), km.tolist(), kn.tolist()))
    assert got == sorted(zip(re.tolist(), rm.tolist(), rn.tolist()))


def test_expert_offsets_on_device(cuda_device):
    for counts in ([], [5], [3, 0, 70, 129], list(range(1000))):
        t = torch.tensor(counts, dtype=torch.int32, device=cuda_device)
        got = mo.expert_offsets_from_recv_counts(t)
        assert got.dtype == torch.int32 and got.is_cuda
        ref = og.expert_offsets_from_recv_counts(counts).astype(np.int32)
        assert np.array_equal(got.cpu().numpy(), ref)
    big = torch.tensor([2 ** 31 + 5, 1, -7], dtype=torch.int64, device=cuda_device)
    got64 = mo.expert_offsets_from_recv_counts(big, dtype=torch.int64)
    assert np.array_equal(got64.cpu().numpy(), og.expert_offsets_from_recv_counts([2 ** 31 + 5, 1, -7]))


def test_status_word_clean_after_valid_calls(cuda_device):
    _lib.check_status(cuda_device, sync=True)
    assert int(_lib.status_word(cuda_device)[0]) == 0


def test_epilogue_row_scale_aux_out_and_dgelu(cuda_device):
    counts = [70, 0, 130, 64]
    a, b, off = gemm_inputs(counts, 256, 384, "bf16", seed=31, w_std=0.05)
    m = a.shape[0]
    g = torch.Generator().manual_seed(32)
    scale = torch.rand(m, generator=g) + 0.5
    aux_in = torch.randn(m, 384, generator=g).to(torch.bfloat16)
    da, db, doff = a.to(cuda_device), b.to(cuda_device), off.to(cuda_device)
    aux_out = torch.empty(m, 384, dtype=torch.bfloat16, device=cuda_device)
    c = mo.grouped_gemm(da, db, doff, activation="gelu", row_scale=scale.to(cuda_device),
                        aux_out=aux_out)
    c2 = mo.grouped_gemm(da, db, doff, activation="dgelu", aux_in=aux_in.to(cuda_device))
    mo.check_status(cuda_device, sync=True)
    want, want_aux, defined = og.grouped_gemm_ex(to_storage(a), to_storage(b), off.numpy(), "bf16",
                                                 "gelu", row_scale=scale.numpy())
    assert_matches_oracle(c, want, defined, "bf16")
    assert_matches_oracle(aux_out, want_aux, defined, "bf16")
    want2, _, _ = og.grouped_gemm_ex(to_storage(a), to_storage(b), off.numpy(), "bf16", "dgelu",
                                     aux_in=to_storage(aux_in))
    assert_matches_oracle(c2, want2, defined, "bf16")


@pytest.mark.parametrize("m,n,num_sms", [(256, 512, 148), (192, 136, 148), (192, 136, 1),
                                         (384, 264, 7), (256, 512, 1)])
def test_wgrad_matches_oracle(cuda_device, m, n, num_sms):
    """num_sms >= 2 runs the CTA-pair kernel (7 -> 3 pairs), 1 the 1-SM kernel."""
    counts = [128, 0, 64, 384, 192]  # 64-row aligned segments, one empty expert
    g = torch.Generator().manual_seed(m + n)
    rows = sum(counts)
    a = torch.randn(rows, m, generator=g).to(torch.bfloat16)
    b = torch.randn(rows, n, generator=g).to(torch.bfloat16)
    off = torch.tensor(og.expert_offsets_from_recv_counts(counts).astype(np.int32))
    c = torch.full((len(counts), m, n), float("nan"), dtype=torch.bfloat16, device=cuda_device)
    lib = _lib.load()
    status = torch.zeros(1, dtype=torch.int32, device=cuda_device)
    da, db, doff = a.to(cuda_device), b.to(cuda_device), off.to(cuda_device)
    rc = lib.moe_grouped_gemm_wgrad(da.data_ptr(), m, db.data_ptr(), n, c.data_ptr(), n, m * n,
                                    doff.data_ptr(), 0, rows, m, n, len(counts),
                                    _lib.MOE_DTYPE_BF16, num_sms, status.data_ptr(),
                                    torch.cuda.current_stream().cuda_stream)
    assert rc == 0
    torch.cuda.synchronize()
    assert int(status.item()) == 0
    want = og.wgrad(to_storage(a), to_storage(b), off.numpy(), "bf16")
    got = to_storage(c.reshape(len(counts) * m, n))
    assert_matches_oracle(torch.from_numpy(got.view(np.int16)).view(torch.bfloat16),
                          want.reshape(len(counts) * m, n), np.ones(len(counts) * m, bool), "bf16")


def test_wgrad_rejects_misaligned_segments(cuda_device):
    rows, m, n = 200, 64, 64
    a = torch.zeros(rows, m, dtype=torch.bfloat16, device=cuda_device)
    b = torch.zeros(rows, n, dtype=torch.bfloat16, device=cuda_device)
    off = torch.tensor([0, 100, 200], dtype=torch.int32, device=cuda_device)
    c = torch.empty(2, m, n, dtype=torch.bfloat16, device=cuda_device)
    status = torch.zeros(1, dtype=torch.int32, device=cuda_device)
    rc = _lib.load().moe_grouped_gemm_wgrad(a.data_ptr(), m, b.data_ptr(), n, c.data_ptr(), n,
                                            m * n, off.data_ptr(), 0, rows, m, n, 2,
                                            _lib.MOE_DTYPE_BF16, 148, status.data_ptr(),
                                            torch.cuda.current_stream().cuda_stream)
    assert rc == 0
    torch.cuda.synchronize()
    assert int(status.item()) == _lib.MOE_ERR_OFFSETS


@pytest.mark.parametrize("num_sms", [148, 1])
def test_epilogue_gelu_save_grad_and_mul_aux(cuda_device, num_sms):
    """GELU with gelu'(v) saved to aux_out, then v * aux_in: the split GELU backward."""
    counts = [70, 0, 130, 64]
    a, b, off = gemm_inputs(counts, 256, 384, "bf16", seed=33, w_std=0.05)
    m = a.shape[0]
    g = torch.Generator().manual_seed(34)
    aux_in = (torch.rand(m, 384, generator=g) * 1.2).to(torch.bfloat16)
    da, db, doff = a.to(cuda_device), b.to(cuda_device), off.to(cuda_device)
    aux_out = torch.empty(m, 384, dtype=torch.bfloat16, device=cuda_device)
    c = mo.grouped_gemm(da, db, doff, activation="gelu_save_grad", aux_out=aux_out, num_sms=num_sms)
    c2 = mo.grouped_gemm(da, db, doff, activation="mul_aux", aux_in=aux_in.to(cuda_device),
                         num_sms=num_sms)
    mo.check_status(cuda_device, sync=True)
    sa, sb = to_storage(a), to_storage(b)
    want, want_aux, defined = og.grouped_gemm_ex(sa, sb, off.numpy(), "bf16", "gelu_save_grad")
    assert_matches_oracle(c, want, defined, "bf16")
    assert_matches_oracle(aux_out, want_aux, defined, "bf16")
    want2, _, _ = og.grouped_gemm_ex(sa, sb, off.numpy(), "bf16", "mul_aux", aux_in=to_storage(aux_in))
    assert_matches_oracle(c2, want2, defined, "bf16")
    with pytest.raises(mo.MoeError):
        mo.grouped_gemm(da, db, doff, activation="gelu_save_grad")  # aux_out is required


def test_operands_on_a_device_that_is_not_current():
    """Operands on cuda:1 while cuda:0 is current run on cuda:1, as torch ops do."""
    if not torch.cuda.is_available() or torch.cuda.device_count() < 2:
        pytest.skip("needs two CUDA devices")
    dev1 = torch.device("cuda", 1)
    if torch.cuda.get_device_capability(dev1)[0] != 10:
        pytest.skip("needs an sm_100 device")
    counts = [40, 0, 300, 129]
    a, b, off = gemm_inputs(counts, 128, 256, "bf16", seed=31)
    with torch.cuda.device(0):
        c = mo.persistent_grouped_gemm(a.to(dev1), b.to(dev1), off.to(dev1), num_sms=148)
        h = mo.grouped_gemm(a.to(dev1), b.to(dev1), off.to(dev1), activation="gelu")
        we, _, _ = mo.tile_list(off.to(dev1), int(off[-1]), 256)
    mo.check_status(dev1, sync=True)
    assert c.device == dev1 and we.device == dev1
    for out, act in ((c, None), (h, "gelu")):
        ref, defined = og.grouped_gemm(to_storage(a), to_storage(b), off.numpy(), "bf16", act)
        assert_matches_oracle(out, ref, defined, "bf16")
