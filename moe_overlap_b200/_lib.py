"""ctypes binding of the in-tree C-ABI library ``libmoe_overlap_b200.so``.

The library is the only compute path: if it is missing or fails to load, every
entry point raises ``RuntimeError``; there is no Python or CPU fallback.

Device-side errors (an expired bounded wait, offsets out of range) are written
by the kernels into a per-device status word that lives in pinned, mapped host
memory.  ``check_status()`` reads it without synchronising; the public entry
points call it before every launch, so an error from an earlier kernel is
raised at the next call (like CUDA's own asynchronous error reporting), and
``check_status(sync=True)`` synchronises first.
"""
from __future__ import annotations

import ctypes
import os
import threading
from pathlib import Path

import torch

LIB_NAME = "libmoe_overlap_b200.so"
LIB_PATH = Path(__file__).resolve().with_name(LIB_NAME)

MOE_OK = 0
MOE_ERR_INVALID_ARG = 1
MOE_ERR_CUDA = 2
MOE_ERR_TIMEOUT = 3
MOE_ERR_OFFSETS = 4
MOE_ERR_UNSUPPORTED = 5
MOE_ERR_CAPACITY = 6

MOE_DTYPE_BF16 = 0
MOE_DTYPE_F16 = 1
MOE_DTYPE_F32 = 2
MOE_ACT_NONE = 0
MOE_ACT_GELU = 1
MOE_ACT_DGELU = 2
MOE_ACT_GELU_SAVE_GRAD = 3
MOE_ACT_MUL_AUX = 4

_c_void_p = ctypes.c_void_p
_i32 = ctypes.c_int32
_i64 = ctypes.c_int64
_u64 = ctypes.c_uint64

# name -> (restype, argtypes); mirrors include/moe_overlap.h
SIGNATURES: dict[str, tuple] = {
    "moe_status_string": (ctypes.c_char_p, [_i32]),
    "moe_abi_version": (_i32, []),
    "moe_grouped_gemm": (
        _i32,
        [
            _c_void_p, _i64,  # a, lda
            _c_void_p, _i64, _i64, _i64,  # b, strides e/k/n
            _c_void_p, _i64,  # c, ldc
            _c_void_p, _i32,  # offsets, offsets_int64
            _i64, _i64, _i64, _i32,  # m_total, k, n, num_experts
            _i32, _i32, _i32, _i32,  # dtype, activation, num_sms, use_atomic_queue
            _c_void_p, _c_void_p, _c_void_p,  # work_counter, status, stream
        ],
    ),
    "moe_grouped_gemm_ex": (
        _i32,
        [
            _c_void_p, _i64,  # a, lda
            _c_void_p, _i64, _i64, _i64,  # b, strides e/k/n
            _c_void_p, _i64,  # c, ldc
            _c_void_p, _i32,  # offsets, offsets_int64
            _i64, _i64, _i64, _i32,  # m_total, k, n, num_experts
            _i32, _i32, _i32, _i32,  # dtype, activation, num_sms, use_atomic_queue
            _c_void_p,  # work_counter
            _c_void_p, _c_void_p, _c_void_p, _i64,  # row_scale, aux_in, aux_out, ld_aux
            _c_void_p, _c_void_p,  # status, stream
        ],
    ),
    "moe_grouped_gemm_wgrad": (
        _i32,
        [
            _c_void_p, _i64, _c_void_p, _i64,  # a, lda, b, ldb
            _c_void_p, _i64, _i64,  # c, ldc, c_stride_e
            _c_void_p, _i32,  # offsets, offsets_int64
            _i64, _i64, _i64, _i32,  # rows_total, m, n, num_experts
            _i32, _i32,  # dtype, num_sms
            _c_void_p, _c_void_p,  # status, stream
        ],
    ),
    "moe_grouped_gemm_noalloc": (
        _i32,
        [
            _c_void_p, _i64,  # a, lda
            _c_void_p, _i64, _i64, _i64,  # b, strides e/k/n
            _c_void_p, _i64,  # c, ldc
            _c_void_p, _i32,  # offsets, offsets_int64
            _i64, _i64, _i64, _i32,  # m_total, k, n, num_experts
            _i32, _i32, _i32,  # dtype, activation, num_sms
            _c_void_p, _c_void_p,  # status, stream
        ],
    ),
    "moe_tile_list": (
        _i32,
        [
            _c_void_p, _i32, _i32, _i64, _i64, _i32, _i32, _i32,
            _c_void_p, _c_void_p, _c_void_p, _i32, _c_void_p, _c_void_p, _c_void_p,
        ],
    ),
    "moe_expert_offsets": (_i32, [_c_void_p, _i32, _i32, _c_void_p, _i32, _c_void_p]),
    "moe_expert_offsets_host": (_i32, [_c_void_p, _i32, _i32, _c_void_p, _i32]),
    # expert-parallel exchange
    "moe_ep_create": (_i32, [_i32, _i32, _i32, _i32, _i32, _i32, _i64, _c_void_p]),
    "moe_ep_destroy": (_i32, [_c_void_p]),
    "moe_ep_buffer": (_i32, [_c_void_p, _c_void_p, _c_void_p]),
    "moe_ep_connect": (_i32, [_c_void_p, _c_void_p]),
    "moe_ep_views": (_i32, [_c_void_p, _i32, _c_void_p]),
    "moe_ep_dispatch_begin": (
        _i32, [_c_void_p, _c_void_p, _c_void_p, _c_void_p, _i32, _i32, _i32, _u64, _c_void_p,
               _c_void_p]),
    "moe_ep_dispatch_scatter": (
        _i32, [_c_void_p, _c_void_p, _c_void_p, _c_void_p, _i32, _i32, _i32, _u64, _i32, _i32,
               _i32, _i32, _u64, _c_void_p, _c_void_p]),
    "moe_ep_dispatch_end": (_i32, [_c_void_p, _i32, _u64, _u64, _c_void_p, _c_void_p]),
    "moe_ep_dispatch": (
        _i32, [_c_void_p, _c_void_p, _c_void_p, _c_void_p, _i32, _i32, _i32, _u64, _i32, _i32,
               _i32, _i32, _u64, _c_void_p, _c_void_p]),
    "moe_ep_dispatch_fp8": (
        _i32, [_c_void_p, _c_void_p, _c_void_p, _c_void_p, _c_void_p,  # ep, x_fp8, scales, idx, w
               _i32, _i32, _i32, _u64, _i32, _i32,  # T, k, slot, epoch, blocks, pad_rows
               _u64, _c_void_p, _c_void_p]),  # wait_ns, status, stream
    "moe_ep_dispatch_fp8_scatter": (
        _i32, [_c_void_p, _c_void_p, _c_void_p, _c_void_p, _c_void_p, _i32, _i32, _i32, _u64, _i32,
               _i32, _u64, _c_void_p, _c_void_p]),
    "moe_fp8_quantize": (
        _i32, [_c_void_p, _i64, _i64, _i32, _c_void_p, _i64, _c_void_p, _i64, _c_void_p]),
    "moe_fp8_dequantize": (
        _i32, [_c_void_p, _i64, _c_void_p, _i64, _c_void_p, _i64, _i32, _c_void_p, _i64,
               _c_void_p]),
    "moe_ep_dispatch_ordered_begin": (
        _i32, [_c_void_p, _c_void_p, _c_void_p, _c_void_p, _i32, _i32, _i32, _u64, _c_void_p,
               _c_void_p]),
    "moe_ep_dispatch_ordered_scatter": (
        _i32, [_c_void_p, _c_void_p, _c_void_p, _c_void_p, _i32, _i32, _i32, _u64, _i32, _i32,
               _u64, _c_void_p, _c_void_p]),
    "moe_ep_dispatch_ordered": (
        _i32, [_c_void_p, _c_void_p, _c_void_p, _c_void_p, _i32, _i32, _i32, _u64, _i32, _i32,
               _u64, _c_void_p, _c_void_p]),
    "moe_ep_expert_gemm": (
        _i32, [_c_void_p, _i32, _c_void_p, _i64, _i64, _i64,  # ep, slot, b, strides e/k/n
               _c_void_p, _i64, _i64, _i32, _i32, _i32, _c_void_p,  # c, ldc, n, act, sms, atomic, ctr
               _u64, _c_void_p, _c_void_p]),  # wait_ns, status, stream
    "moe_ep_dispatch_cached_begin": (_i32, [_c_void_p, _i32, _u64, _c_void_p]),
    "moe_ep_dispatch_cached_scatter": (
        _i32, [_c_void_p, _c_void_p, _c_void_p, _c_void_p, _i32, _i32, _i32, _i32, _u64, _i32,
               _i32, _i32, _u64, _c_void_p, _c_void_p]),
    "moe_ep_dispatch_cached": (
        _i32, [_c_void_p, _c_void_p, _c_void_p, _c_void_p, _i32, _i32, _i32, _i32, _u64, _i32,
               _i32, _i32, _u64, _c_void_p, _c_void_p]),
    "moe_ep_topk_weight_grad": (
        _i32, [_c_void_p, _c_void_p, _c_void_p, _i32, _i32, _i32, _c_void_p, _i32, _c_void_p]),
    "moe_ep_combine_begin": (_i32, [_c_void_p, _i32, _u64, _c_void_p]),
    "moe_ep_combine_end": (
        _i32, [_c_void_p, _c_void_p, _c_void_p, _i32, _i32, _i32, _u64, _i32, _c_void_p, _i32,
               _u64, _c_void_p, _c_void_p]),
    "moe_ep_combine": (
        _i32, [_c_void_p, _c_void_p, _c_void_p, _i32, _i32, _i32, _u64, _i32, _c_void_p, _i32,
               _u64, _c_void_p, _c_void_p]),
    "moe_ep_set_device_epoch": (_i32, [_c_void_p, ctypes.c_uint64, _c_void_p]),
    "moe_ep_push_gemm": (
        _i32,
        [_c_void_p, _c_void_p, _i64, _c_void_p, _i64, _i64, _i64,  # ep, a, lda, b, strides e/k/n
         _i64, _i64, _i32, _i32, _i32, _c_void_p,  # m_total, k, dtype, num_sms, atomic, counter
         _i32, ctypes.c_uint64, _c_void_p, _c_void_p],  # slot, epoch, status, stream
    ),
    "moe_ep_combine_pushed": (
        _i32,
        [_c_void_p, _c_void_p, _c_void_p, _i32, _i32, _i32, ctypes.c_uint64,  # ep, idx, w, T, k, slot, epoch
         _i32, _c_void_p, _i32, ctypes.c_uint64, _c_void_p, _c_void_p],  # weighted, out, blocks, wait, status, stream
    ),
    "moe_router_topk": (
        _i32,
        [_c_void_p, _i32, _c_void_p, _i32, _i32, _i32, _i32,  # logits, dtype, bias, T, E, k, renorm
         _c_void_p, _c_void_p, _c_void_p, _c_void_p],  # probs, idx, weights, stream
    ),
    "moe_router_topk_backward": (
        _i32,
        [_c_void_p, _c_void_p, _c_void_p, _i32, _i32, _i32, _i32,  # probs, idx, dw, T, E, k, renorm
         _c_void_p, _c_void_p],  # grad_logits, stream
    ),
    "moe_ep_dispatch_layout": (
        _i32, [_c_void_p, _i32, _i32, _i32, _i32, _c_void_p, _c_void_p, _c_void_p, _c_void_p]),
    "moe_ipc_export": (_i32, [_c_void_p, _c_void_p]),
    "moe_ipc_import": (_i32, [_c_void_p, _c_void_p]),
    "moe_ipc_close": (_i32, [_c_void_p]),
}

_lock = threading.Lock()
_lib: ctypes.CDLL | None = None
_status_words: dict[int, torch.Tensor] = {}


class MoeError(RuntimeError):
    """A status code returned by the library or recorded by one of its kernels."""

    def __init__(self, code: int, where: str):
        self.code = code
        super().__init__(f"{where}: {status_string(code)} (status {code})")


def load() -> ctypes.CDLL:
    """Loads the library once and declares every exported signature."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is None:
            if not LIB_PATH.exists():
                raise RuntimeError(
                    f"{LIB_NAME} is not built (expected at {LIB_PATH}); "
                    "run `python -m moe_overlap_b200.build`"
                )
            lib = ctypes.CDLL(str(LIB_PATH), mode=os.RTLD_NOW | os.RTLD_LOCAL)
            for name, (restype, argtypes) in SIGNATURES.items():
                fn = getattr(lib, name)
                fn.restype = restype
                fn.argtypes = argtypes
            _lib = lib
    return _lib


def status_string(code: int) -> str:
    return load().moe_status_string(int(code)).decode()


def status_word(device: torch.device) -> torch.Tensor:
    """Pinned host int32 the kernels on ``device`` write their error code into."""
    idx = device.index if device.index is not None else torch.cuda.current_device()
    w = _status_words.get(idx)
    if w is None:
        with _lock:
            w = _status_words.get(idx)
            if w is None:
                w = torch.zeros(1, dtype=torch.int32, pin_memory=True)
                _status_words[idx] = w
    return w


def check_status(device: torch.device | None = None, sync: bool = False) -> None:
    """Raises MoeError if a kernel on ``device`` recorded an error (and clears it)."""
    if device is None:
        device = torch.device("cuda", torch.cuda.current_device())
    if sync:
        torch.cuda.synchronize(device)
    w = status_word(device)
    code = int(w[0])
    if code != 0:
        w.zero_()
        raise MoeError(code, "device-side error from an earlier moe_overlap_b200 kernel")


def check_call(code: int, where: str) -> None:
    if code != MOE_OK:
        raise MoeError(code, where)


def stream_handle(device: torch.device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def sync_check_enabled() -> bool:
    """MOE_B200_SYNC_CHECK=1 synchronises and checks the status after every call."""
    return os.environ.get("MOE_B200_SYNC_CHECK", "0") not in ("", "0")
