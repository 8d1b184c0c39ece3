"""CPU-only checks of the C-ABI library and the host-side mirror of the reference API.

No kernel is launched here: the library must load without a GPU, export every
entry point that include/*.h declares, reject bad arguments on the host with
the documented status codes, and the Python layer must raise the reference's
exceptions (src/triton_grouped_gemm.py:347-360, 383-384).
"""
import ctypes
import re
from pathlib import Path

import pytest
import torch

import moe_overlap_b200 as mo
from moe_overlap_b200 import _lib

HEADERS = sorted((Path(__file__).resolve().parents[1] / "include").glob("*.h"))


def declared_symbols() -> list[str]:
    names = []
    for h in HEADERS:
        text = h.read_text()
        names += re.findall(r"^MOE_API\s+[\w\s\*]+?\b(moe_\w+)\s*\(", text, flags=re.M)
    return names


def test_headers_declare_entry_points():
    names = declared_symbols()
    assert "moe_grouped_gemm" in names and "moe_expert_offsets" in names
    assert len(names) == len(set(names))


@pytest.mark.parametrize("name", declared_symbols())
def test_library_exports_every_declared_symbol(name):
    lib = ctypes.CDLL(str(_lib.LIB_PATH))
    assert hasattr(lib, name), f"{name} declared in include/ but not exported"
    assert name in _lib.SIGNATURES, f"{name} has no ctypes signature in _lib.SIGNATURES"


def test_abi_version_and_status_strings():
    lib = _lib.load()
    assert lib.moe_abi_version() == 1
    for code in range(7):
        assert _lib.status_string(code)
    assert _lib.status_string(99) == "unknown status"


def _gemm_call(**kw):
    args = dict(a=16, lda=64, b=16, se=64 * 64, sk=64, sn=1, c=16, ldc=64, off=16, off64=0,
                m=10, k=64, n=64, e=1, dtype=0, act=0, sms=148, atomic=0, counter=None,
                status=None, stream=None)
    args.update(kw)
    return _lib.load().moe_grouped_gemm(*args.values())


@pytest.mark.parametrize(
    "kw",
    [
        dict(dtype=7),                 # unknown dtype
        dict(act=9),                   # unknown activation
        dict(m=-1),                    # negative size
        dict(e=2000),                  # more experts than the scheduler's smem table
        dict(n=12, ldc=16),            # n not a multiple of 8
        dict(k=12, lda=16),            # k not a multiple of 8
        dict(c=18),                    # misaligned output
        dict(a=24),                    # misaligned A
        dict(sn=2, sk=2),              # B neither N-major nor K-major
        dict(atomic=1, counter=None),  # atomic queue without a counter
        dict(off=None),                # no offsets
    ],
)
def test_grouped_gemm_rejects_bad_arguments_on_host(kw):
    code = _gemm_call(**kw)
    assert code in (_lib.MOE_ERR_INVALID_ARG, _lib.MOE_ERR_UNSUPPORTED), code


def test_grouped_gemm_empty_output_is_a_no_op():
    assert _gemm_call(m=0) == _lib.MOE_OK
    assert _gemm_call(n=0) == _lib.MOE_OK


def test_tile_list_and_offsets_reject_bad_arguments():
    lib = _lib.load()
    assert lib.moe_tile_list(None, 0, 4, 10, 10, 128, 128, 0, None, None, None, 0, 16, None,
                             None) == _lib.MOE_ERR_INVALID_ARG
    assert lib.moe_tile_list(16, 0, 4, 10, 10, 128, 128, 2, None, None, None, 0, 16, None,
                             None) == _lib.MOE_ERR_INVALID_ARG
    assert lib.moe_expert_offsets(None, 0, 4, 16, 0, None) == _lib.MOE_ERR_INVALID_ARG
    assert lib.moe_expert_offsets_host(None, 0, 3, None, 0) == _lib.MOE_ERR_INVALID_ARG


def _cpu_args():
    a = torch.zeros(8, 16, dtype=torch.bfloat16)
    b = torch.zeros(2, 16, 8, dtype=torch.bfloat16)
    off = torch.tensor([0, 4, 8], dtype=torch.int32)
    return a, b, off


def test_persistent_grouped_gemm_requires_cuda_tensors():
    a, b, off = _cpu_args()
    with pytest.raises(ValueError, match="requires CUDA tensors"):
        mo.persistent_grouped_gemm(a, b, off)


def test_host_mirror_error_messages_match_reference(monkeypatch):
    """Validation order and messages of src/triton_grouped_gemm.py:347-360."""
    from moe_overlap_b200 import gemm as gg

    class FakeCuda:
        type = "cuda"

        def __eq__(self, other):
            return isinstance(other, FakeCuda)

    class T:
        def __init__(self, shape, dtype=torch.bfloat16, device=None):
            self.shape, self.dtype = shape, dtype
            self.device = device or FakeCuda()

        def dim(self):
            return len(self.shape)

        def size(self, i):
            return self.shape[i]

        def numel(self):
            n = 1
            for s in self.shape:
                n *= s
            return n

    a, b, off = T((8, 16)), T((2, 16, 8)), T((3,), torch.int32)
    cases = [
        ((T((8,)), b, off), "Shapes must be"),
        ((T((8, 12)), b, off), "K dimension mismatch"),
        ((a, b, T((4,), torch.int32)), r"expert_offsets must have shape \[num_experts \+ 1\]"),
        ((a, b, T((3,), torch.int32, device=torch.device("cpu"))), "same device"),
        ((T((8, 16), torch.float32), T((2, 16, 8), torch.float32), off), "bf16/fp16"),
        ((a, T((2, 16, 8), torch.float16), off), "should match a_cat dtype"),
    ]
    for args, msg in cases:
        with pytest.raises(ValueError, match=msg):
            gg.persistent_grouped_gemm(*args)
    with pytest.raises(ValueError, match="work_counter must be int32"):
        gg.persistent_grouped_gemm(a, b, off, work_counter=T((2,), torch.int32))


def test_library_missing_fails_loudly(monkeypatch, tmp_path):
    monkeypatch.setattr(_lib, "_lib", None)
    monkeypatch.setattr(_lib, "LIB_PATH", tmp_path / "missing.so")
    with pytest.raises(RuntimeError, match="is not built"):
        _lib.load()


def test_router_entry_points_reject_bad_arguments_on_host():
    """Argument checks that return before any CUDA call (runs without a GPU)."""
    lib = _lib.load()
    bf16 = _lib.MOE_DTYPE_BF16
    # more than 256 experts, top_k above the experts, top_k above 16, bad dtype
    assert lib.moe_router_topk(None, bf16, None, 4, 300, 2, 0, None, None, None, None) == \
        _lib.MOE_ERR_INVALID_ARG
    assert lib.moe_router_topk(None, bf16, None, 4, 8, 9, 0, None, None, None, None) == \
        _lib.MOE_ERR_INVALID_ARG
    assert lib.moe_router_topk(None, bf16, None, 4, 64, 17, 0, None, None, None, None) == \
        _lib.MOE_ERR_INVALID_ARG
    assert lib.moe_router_topk(None, 7, None, 4, 8, 2, 0, None, None, None, None) == \
        _lib.MOE_ERR_INVALID_ARG
    # missing buffers with tokens to route
    assert lib.moe_router_topk(None, bf16, None, 4, 8, 2, 0, None, None, None, None) == \
        _lib.MOE_ERR_INVALID_ARG
    assert lib.moe_router_topk_backward(None, None, None, 4, 8, 2, 1, None, None) == \
        _lib.MOE_ERR_INVALID_ARG
    # no tokens: nothing to do
    assert lib.moe_router_topk(None, bf16, None, 0, 8, 2, 0, None, None, None, None) == _lib.MOE_OK
    assert lib.moe_router_topk_backward(None, None, None, 0, 8, 2, 0, None, None) == _lib.MOE_OK


def test_grouped_gemm_activation_codes_checked_on_host():
    """GELU_SAVE_GRAD needs aux_out and MUL_AUX/DGELU need aux_in; the plain entry point
    takes none of them; unknown codes are rejected - all before any CUDA call."""
    lib = _lib.load()
    common = (None, 64, None, 64 * 64, 64, 1, None, 64, None, 0, 64, 64, 64, 1,
              _lib.MOE_DTYPE_BF16)
    for act in (_lib.MOE_ACT_DGELU, _lib.MOE_ACT_GELU_SAVE_GRAD, _lib.MOE_ACT_MUL_AUX, 5, -1):
        assert lib.moe_grouped_gemm(*common, act, 1, 0, None, None, None) == \
            _lib.MOE_ERR_INVALID_ARG, act
    ex_tail = (None, None, None, None, 64, None, None)
    for act in (_lib.MOE_ACT_DGELU, _lib.MOE_ACT_MUL_AUX, _lib.MOE_ACT_GELU_SAVE_GRAD):
        assert lib.moe_grouped_gemm_ex(*common, act, 1, 0, *ex_tail) == _lib.MOE_ERR_INVALID_ARG, act


def test_cached_dispatch_entry_points_reject_bad_arguments_on_host():
    """Without an endpoint, or with the source slot equal to the target slot, the
    cached re-dispatch returns MOE_ERR_INVALID_ARG before any CUDA call."""
    lib = _lib.load()
    bad = _lib.MOE_ERR_INVALID_ARG
    assert lib.moe_ep_dispatch_cached_begin(None, 0, 1, None) == bad
    for src_slot, slot in ((0, 1), (1, 1), (2, 0), (0, -1)):
        assert lib.moe_ep_dispatch_cached_scatter(None, None, None, None, 4, 2, src_slot, slot, 1, 8,
                                                  0, 0, 10**9, None, None) == bad, (src_slot, slot)
        assert lib.moe_ep_dispatch_cached(None, None, None, None, 4, 2, src_slot, slot, 1, 8, 0, 0,
                                          10**9, None, None) == bad, (src_slot, slot)


def test_fp8_and_ordered_entry_points_reject_bad_arguments_on_host():
    """The FP8 payload, the expert-ordered dispatch and its waiting GEMM check their
    arguments (no endpoint, bad slot, hidden size, alignment, activation) before any
    CUDA call and return MOE_ERR_INVALID_ARG."""
    lib = _lib.load()
    bad = _lib.MOE_ERR_INVALID_ARG
    assert lib.moe_ep_dispatch_fp8(None, None, None, None, None, 4, 2, 0, 1, 8, 0, 10**9, None,
                                   None) == bad
    assert lib.moe_ep_dispatch_fp8_scatter(None, None, None, None, None, 4, 2, 0, 1, 8, 0, 10**9,
                                           None, None) == bad
    assert lib.moe_ep_dispatch_ordered(None, None, None, None, 4, 2, 0, 1, 8, 0, 10**9, None,
                                       None) == bad
    assert lib.moe_ep_dispatch_ordered_begin(None, None, None, None, 4, 2, 0, 1, None, None) == bad
    assert lib.moe_ep_dispatch_ordered_scatter(None, None, None, None, 4, 2, 0, 1, 8, 0, 10**9,
                                               None, None) == bad
    for slot, act in ((0, _lib.MOE_ACT_NONE), (2, _lib.MOE_ACT_NONE), (0, _lib.MOE_ACT_DGELU)):
        assert lib.moe_ep_expert_gemm(None, slot, None, 0, 0, 0, None, 0, 64, act, 148, 1, None,
                                      10**9, None, None) == bad
    # quantise / dequantise: hidden not a multiple of 128, strides too small, misaligned
    assert lib.moe_fp8_quantize(None, 200, 4, 200, None, 200, None, 2, None) == bad
    assert lib.moe_fp8_quantize(None, 100, 4, 256, None, 256, None, 2, None) == bad
    assert lib.moe_fp8_quantize(4, 256, 4, 256, 16, 256, 32, 2, None) == bad  # x not 8-aligned
    assert lib.moe_fp8_dequantize(None, 256, None, 1, None, 4, 256, None, 256, None) == bad
    assert lib.moe_fp8_dequantize(None, 200, None, 2, None, 4, 200, None, 200, None) == bad
    # zero rows is a no-op
    assert lib.moe_fp8_quantize(None, 256, 0, 256, None, 256, None, 2, None) == _lib.MOE_OK
    assert lib.moe_fp8_dequantize(None, 256, None, 2, None, 0, 256, None, 256, None) == _lib.MOE_OK


C_CLIENT = r"""
#include <stdio.h>
#include <string.h>
#include "moe_overlap.h"
int main(void) {
  int32_t counts[4] = {3, 0, 5, 2};
  int64_t off[5];
  if (moe_expert_offsets_host(counts, 0, 4, off, 1) != MOE_OK) return 1;
  if (off[0] != 0 || off[1] != 3 || off[2] != 3 || off[3] != 8 || off[4] != 10) return 2;
  if (moe_abi_version() != MOE_ABI_VERSION) return 3;
  if (strlen(moe_status_string(MOE_ERR_TIMEOUT)) == 0) return 4;
  if (moe_ep_dispatch_cached_begin(NULL, 0, 1, NULL) != MOE_ERR_INVALID_ARG) return 5;
  puts("ok");
  return 0;
}
"""


def test_header_is_plain_c_and_a_c_program_links_the_library(tmp_path):
    """A C host (no C++, no torch) compiles against include/moe_overlap.h with
    -std=c99 -pedantic -Werror, links the library and calls its host-side entry points."""
    import shutil
    import subprocess

    gcc = shutil.which("gcc")
    if gcc is None:
        pytest.skip("gcc not available")
    repo = Path(__file__).resolve().parents[1]
    _lib.load()  # fails loudly if the library is not built
    lib = _lib.LIB_PATH
    src = tmp_path / "client.c"
    src.write_text(C_CLIENT)
    exe = tmp_path / "client"
    r = subprocess.run([gcc, "-std=c99", "-Wall", "-Wextra", "-pedantic", "-Werror",
                        "-I", str(repo / "include"), str(src), "-L", str(lib.parent),
                        "-l" + lib.stem[3:], f"-Wl,-rpath,{lib.parent}", "-o", str(exe)],
                       capture_output=True, text=True)
    assert r.returncode == 0, r.stderr
    run = subprocess.run([str(exe)], capture_output=True, text=True, timeout=60)
    assert run.returncode == 0 and run.stdout.strip() == "ok", (run.returncode, run.stdout, run.stderr)


def test_extended_gemm_entry_points_refuse_host_tensors():
    """grouped_gemm / grouped_gemm_wgrad hand raw pointers to the kernels: a CPU
    operand (a host pointer on the GPU) is refused on the host instead."""
    from moe_overlap_b200 import gemm as gg

    a, b, off = _cpu_args()
    with pytest.raises(ValueError, match="must be CUDA tensors"):
        gg.grouped_gemm(a, b, off)
    with pytest.raises(ValueError, match="must be CUDA tensors"):
        gg.grouped_gemm_wgrad(torch.zeros(64, 8, dtype=torch.bfloat16),
                              torch.zeros(64, 8, dtype=torch.bfloat16), torch.tensor([0, 64]))
    cuda0 = torch.device("cuda", 0)
    with pytest.raises(ValueError, match=r"aux_in must be on cuda:0, not cpu"):
        gg._require_on_device(cuda0, out=None, aux_in=torch.zeros(2))
    gg._require_on_device(cuda0, out=None)  # absent operands are fine
    with pytest.raises(ValueError, match="must be CUDA tensors"):
        gg.tile_list(off, 8, 8)


def test_dispatcher_refuses_operands_off_its_device():
    """The exchange kernels take raw pointers; the dispatcher refuses a tensor that is
    not on its GPU before anything is enqueued (checked here without a GPU)."""
    from moe_overlap_b200.deep_ep_comm import DeepEPDispatcher

    d = DeepEPDispatcher.__new__(DeepEPDispatcher)  # no buffers needed for the check
    d.device = torch.device("cuda", 0)
    with pytest.raises(ValueError, match=r"x must be on cuda:0, not cpu"):
        d._require_on_device(x=torch.zeros(4, 8), topk_idx=None)
    d._require_on_device(topk_weights=None)
    from moe_overlap_b200.ep import Endpoint

    e = Endpoint.__new__(Endpoint)
    e.device = torch.device("cuda", 0)
    with pytest.raises(ValueError, match=r"exchange operands must be on cuda:0, not cpu"):
        e.dispatch_begin(torch.zeros(4, 8), torch.zeros(4, 2, dtype=torch.int64),
                         torch.zeros(4, 2), 0, 1, None)
