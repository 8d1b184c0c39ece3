"""FP8 (e4m3, per-128-column scales) dispatch payload.

DeepEP's dispatch carries a token either as a bf16 row or as the pair
(x_fp8 [T, H] float8_e4m3fn, x_scales [T, H/128] float32)
(thirdParty/DeepEP/deep_ep/buffer.py:338-342), which halves the bytes that
cross NVLink.  ``quantize_fp8`` and ``dequantize_fp8`` make and undo that pair
on the GPU exactly as DeepEP's helpers define it (tests/utils.py:50-75); the
exchange itself is ``DeepEPDispatcher.dispatch_fp8``.
"""
from __future__ import annotations

from typing import Optional

import torch

from . import _lib

GROUP = 128


def _require_cuda(**tensors) -> torch.device:
    dev = None
    for name, t in tensors.items():
        if t is None:
            continue
        if t.device.type != "cuda":
            raise ValueError(f"{name} must be a CUDA tensor")
        if dev is not None and t.device != dev:
            raise ValueError(f"{name} must be on {dev}, not {t.device}")
        dev = t.device
    return dev


def quantize_fp8(x: torch.Tensor, out: Optional[torch.Tensor] = None,
                 out_scales: Optional[torch.Tensor] = None) -> tuple[torch.Tensor, torch.Tensor]:
    """bf16 ``[T, H]`` -> (e4m3 ``[T, H]``, float32 scales ``[T, H/128]``).

    Per row and 128-column group: amax = max|x| clamped to 1e-4,
    q = e4m3(x * (1/amax * 448)) (nearest even, saturating), scale = amax / 448.
    """
    if x.dtype != torch.bfloat16 or x.dim() != 2:
        raise ValueError("quantize_fp8 expects a bf16 [T, H] tensor")
    t, h = x.shape
    if h % GROUP != 0:
        raise ValueError(f"hidden size ({h}) must be a multiple of {GROUP}")
    device = _require_cuda(x=x, out=out, out_scales=out_scales)
    xc = x if (x.stride(1) == 1 and x.stride(0) % 4 == 0 and x.data_ptr() % 8 == 0) else x.contiguous()
    if out is None:
        out = torch.empty((t, h), dtype=torch.float8_e4m3fn, device=device)
    if out_scales is None:
        out_scales = torch.empty((t, h // GROUP), dtype=torch.float32, device=device)
    if out.shape != (t, h) or out.dtype != torch.float8_e4m3fn or out.stride(1) != 1:
        raise ValueError("out must be float8_e4m3fn [T, H] with unit column stride")
    if out_scales.shape != (t, h // GROUP) or out_scales.dtype != torch.float32 or \
            out_scales.stride(1) != 1:
        raise ValueError("out_scales must be float32 [T, H/128] with unit column stride")
    with torch.cuda.device(device):
        rc = _lib.load().moe_fp8_quantize(xc.data_ptr(), xc.stride(0), t, h, out.data_ptr(),
                                          out.stride(0), out_scales.data_ptr(),
                                          out_scales.stride(0), _lib.stream_handle(device))
    _lib.check_call(rc, "moe_fp8_quantize")
    return out, out_scales


def dequantize_fp8(x_fp8: torch.Tensor, scales: torch.Tensor, out: Optional[torch.Tensor] = None,
                   rows: Optional[torch.Tensor] = None) -> torch.Tensor:
    """(e4m3 ``[T, H]``, float32 scales ``[T, H/128]``) -> bf16 ``[T, H]``: bf16(q * scale).

    ``rows`` (a device int32 scalar tensor, e.g. the last of a dispatch's
    ``expert_offsets``) limits the conversion to the first ``rows`` rows, read on
    the device; rows past it are left as they were in ``out``.
    """
    if x_fp8.dtype != torch.float8_e4m3fn or x_fp8.dim() != 2:
        raise ValueError("dequantize_fp8 expects a float8_e4m3fn [T, H] tensor")
    t, h = x_fp8.shape
    if h % GROUP != 0 or scales.shape != (t, h // GROUP) or scales.dtype != torch.float32:
        raise ValueError("scales must be float32 [T, H/128] and H a multiple of 128")
    device = _require_cuda(x_fp8=x_fp8, scales=scales, out=out, rows=rows)
    if out is None:
        out = torch.empty((t, h), dtype=torch.bfloat16, device=device)
    if out.shape != (t, h) or out.dtype != torch.bfloat16 or out.stride(1) != 1 or \
            out.stride(0) % 8 != 0 or out.data_ptr() % 16 != 0:
        raise ValueError("out must be a bf16 [T, H] tensor with 16-byte aligned rows")
    if x_fp8.stride(1) != 1 or x_fp8.stride(0) % 8 != 0 or x_fp8.data_ptr() % 8 != 0:
        x_fp8 = x_fp8.contiguous()
    if scales.stride(1) != 1:
        scales = scales.contiguous()
    if rows is not None and (rows.dtype != torch.int32 or rows.numel() != 1):
        raise ValueError("rows must be a one-element int32 tensor")
    with torch.cuda.device(device):
        rc = _lib.load().moe_fp8_dequantize(x_fp8.data_ptr(), x_fp8.stride(0), scales.data_ptr(),
                                            scales.stride(0),
                                            rows.data_ptr() if rows is not None else None, t, h,
                                            out.data_ptr(), out.stride(0),
                                            _lib.stream_handle(device))
    _lib.check_call(rc, "moe_fp8_dequantize")
    return out
