"""Grouped GEMM entry points with the call surface of src/triton_grouped_gemm.py.

``persistent_grouped_gemm``, ``expert_offsets_from_recv_counts`` and
``reference_grouped_gemm`` keep the reference's names, arguments, defaults,
return values and error behaviour; the compute runs in the sm_100a kernels of
``libmoe_overlap_b200.so`` (tcgen05/TMEM persistent grouped GEMM, on-device
tile scheduler).  There is no Triton and no CPU fallback.
"""
from __future__ import annotations

from typing import List, Optional, Union

import torch
import torch.nn.functional as F

from . import _lib

__all__ = [
    "persistent_grouped_gemm",
    "grouped_gemm",
    "grouped_gemm_wgrad",
    "expert_offsets_from_recv_counts",
    "reference_grouped_gemm",
    "tile_list",
]

_DTYPE_CODE = {torch.bfloat16: _lib.MOE_DTYPE_BF16, torch.float16: _lib.MOE_DTYPE_F16}
_ACT_CODE = {None: _lib.MOE_ACT_NONE, "none": _lib.MOE_ACT_NONE, "gelu": _lib.MOE_ACT_GELU,
             "dgelu": _lib.MOE_ACT_DGELU, "gelu_save_grad": _lib.MOE_ACT_GELU_SAVE_GRAD,
             "mul_aux": _lib.MOE_ACT_MUL_AUX}


def _require_on_device(device: torch.device, **tensors) -> None:
    """Every given tensor must be a CUDA tensor on ``device``: the kernels take raw
    pointers, and a host pointer handed to one would fault the GPU."""
    if device.type != "cuda":
        raise ValueError("grouped GEMM operands must be CUDA tensors")
    for name, t in tensors.items():
        if t is not None and t.device != device:
            raise ValueError(f"{name} must be on {device}, not {t.device}")


def _aligned(t: torch.Tensor) -> bool:
    return t.data_ptr() % 16 == 0


def _prepare_a(a: torch.Tensor, k_pad: int) -> torch.Tensor:
    if k_pad:
        return F.pad(a, (0, k_pad))
    if a.stride(1) != 1 or a.stride(0) % 8 != 0 or a.stride(0) < a.size(1) or not _aligned(a):
        return a.contiguous()
    return a


def _prepare_b(b: torch.Tensor, k_pad: int, n_pad: int) -> torch.Tensor:
    if k_pad or n_pad:
        return F.pad(b, (0, n_pad, 0, k_pad)).contiguous()
    e, k, n = b.shape
    n_major = b.stride(2) == 1 and b.stride(1) % 8 == 0 and b.stride(1) >= n
    k_major = b.stride(1) == 1 and b.stride(2) % 8 == 0 and b.stride(2) >= k
    e_ok = e == 1 or (b.stride(0) % 8 == 0 and b.stride(0) > 0)
    if not (n_major or k_major) or not e_ok or not _aligned(b):
        return b.contiguous()
    return b


def grouped_gemm(
    a_cat: torch.Tensor,
    b_expert: torch.Tensor,
    expert_offsets: torch.Tensor,
    *,
    out: Optional[torch.Tensor] = None,
    activation: Optional[str] = None,
    num_sms: Optional[int] = None,
    use_atomic_queue: bool = False,
    work_counter: Optional[torch.Tensor] = None,
    row_scale: Optional[torch.Tensor] = None,
    aux_in: Optional[torch.Tensor] = None,
    aux_out: Optional[torch.Tensor] = None,
) -> torch.Tensor:
    """``out[off[e]:off[e+1]] = act(a_cat[off[e]:off[e+1]] @ b_expert[e])`` on the GPU.

    Optional epilogue operands: ``row_scale`` (float32 ``[M]``, multiplies each
    row of the product), ``aux_out`` (``[M, N]``, receives the product before
    the activation) and ``aux_in`` (``[M, N]``; with ``activation="dgelu"`` the
    result is the product times gelu'(aux_in), the fused GELU backward).
    ``activation="gelu_save_grad"`` writes GELU(product) and puts gelu'(product)
    in ``aux_out`` (one erf per element); ``activation="mul_aux"`` multiplies the
    product by ``aux_in`` (the backward against that saved derivative).

    The extended entry point behind ``persistent_grouped_gemm``: optional fused
    exact GELU (``activation="gelu"``), caller-provided output, and ``num_sms``
    defaulting to every SM of the device.  ``b_expert`` may be N-major (the
    reference layout, ``[E, K, N]`` contiguous) or a K-major view such as
    ``w.transpose(1, 2)`` of ``[E, N, K]`` weights; no copy is made for either.
    """
    device = a_cat.device
    _require_on_device(device, b_expert=b_expert, expert_offsets=expert_offsets, out=out,
                       work_counter=work_counter, row_scale=row_scale, aux_in=aux_in, aux_out=aux_out)
    m_total, k_size = a_cat.shape
    num_experts, _, n_size = b_expert.shape
    dtype_code = _DTYPE_CODE[a_cat.dtype]
    act_code = _ACT_CODE[activation]

    k_pad = (-k_size) % 8
    n_pad = (-n_size) % 8
    a_use = _prepare_a(a_cat, k_pad)
    b_use = _prepare_b(b_expert, k_pad, n_pad)
    n_use = n_size + n_pad

    if out is None:
        out = torch.empty((m_total, n_size), device=device, dtype=a_cat.dtype)
    c_use = out
    if n_pad or out.stride(1) != 1 or out.stride(0) % 8 != 0 or not _aligned(out):
        c_use = torch.empty((m_total, n_use), device=device, dtype=a_cat.dtype)

    if expert_offsets.dtype == torch.int64:
        offs, offs64 = expert_offsets.contiguous(), 1
    elif expert_offsets.dtype == torch.int32:
        offs, offs64 = expert_offsets.contiguous(), 0
    else:
        offs, offs64 = expert_offsets.to(torch.int32).contiguous(), 0

    if num_sms is None or num_sms <= 0:
        num_sms = torch.cuda.get_device_properties(device).multi_processor_count
    counter_ptr = 0
    if use_atomic_queue:
        if work_counter is None:
            work_counter = torch.empty(1, device=device, dtype=torch.int32)
        counter_ptr = work_counter.data_ptr()

    ld_aux = 0
    for t in (aux_in, aux_out):
        if t is not None:
            if (t.shape != (m_total, n_size) or t.dtype != a_cat.dtype or t.stride(1) != 1
                    or n_pad or t.data_ptr() % 16 != 0 or t.stride(0) % 8 != 0):
                raise ValueError("aux tensors must be [M, N] in the input dtype, 16-byte aligned rows")
            if ld_aux and t.stride(0) != ld_aux:
                raise ValueError("aux_in and aux_out must share a row stride")
            ld_aux = t.stride(0)
    if row_scale is not None and (row_scale.dtype != torch.float32 or row_scale.numel() < m_total
                                  or not row_scale.is_contiguous()):
        raise ValueError("row_scale must be a contiguous float32 tensor of M entries")
    lib = _lib.load()
    _lib.check_status(device)
    status = _lib.status_word(device)
    # The C layer reads the SM count and architecture of the current device and
    # launches there: make the operands' device current for the call.
    with torch.cuda.device(device):
        rc = lib.moe_grouped_gemm_ex(
            a_use.data_ptr(), a_use.stride(0),
            b_use.data_ptr(), b_use.stride(0), b_use.stride(1), b_use.stride(2),
            c_use.data_ptr(), c_use.stride(0),
            offs.data_ptr(), offs64,
            m_total, k_size + k_pad, n_use, num_experts,
            dtype_code, act_code, int(num_sms), 1 if use_atomic_queue else 0,
            counter_ptr,
            row_scale.data_ptr() if row_scale is not None else None,
            aux_in.data_ptr() if aux_in is not None else None,
            aux_out.data_ptr() if aux_out is not None else None,
            ld_aux, status.data_ptr(), _lib.stream_handle(device),
        )
    _lib.check_call(rc, "moe_grouped_gemm_ex")
    if c_use is not out:
        out.copy_(c_use[:, :n_size])
    if _lib.sync_check_enabled():
        _lib.check_status(device, sync=True)
    return out


def persistent_grouped_gemm(
    a_cat: torch.Tensor,
    b_expert: torch.Tensor,
    expert_offsets: torch.Tensor,
    num_sms: int = 24,
    block_m: int = 128,
    block_n: int = 128,
    block_k: int = 32,
    use_atomic_queue: bool = True,
    work_counter: Optional[torch.Tensor] = None,
    num_warps: int = 8,
    num_stages: int = 3,
) -> torch.Tensor:
    """Grouped GEMM with persistent workers (striped or atomic dequeue).

    Same contract as src/triton_grouped_gemm.py:326-443: returns a new
    ``[M, N]`` tensor whose rows ``off[e]:off[e+1]`` hold ``a_cat[rows] @
    b_expert[e]`` (fp32 accumulation, rounded to the input dtype); the whole
    output is zero when no expert has rows.  ``num_sms`` is the persistent grid
    size; ``use_atomic_queue`` selects the global atomic tile queue, whose
    counter (``work_counter``, int32 ``[1]``) is reset by this call.  The
    Triton tuning knobs ``block_m/block_n/block_k/num_warps/num_stages`` are
    accepted for compatibility; the tile shape is fixed: 256x256 per CTA pair
    (tcgen05 cta_group::2 UMMA 256x256x16, six TMA stages of 64-deep k-blocks),
    or 128x256 on the one-SM kernel used for a grid of one SM.
    """
    if a_cat.device.type != "cuda" or b_expert.device.type != "cuda":
        raise ValueError("persistent_grouped_gemm requires CUDA tensors.")
    if a_cat.dim() != 2 or b_expert.dim() != 3:
        raise ValueError("Shapes must be a_cat [M, K], b_expert [E, K, N].")
    if a_cat.size(1) != b_expert.size(1):
        raise ValueError("K dimension mismatch between a_cat and b_expert.")
    if expert_offsets.numel() != b_expert.size(0) + 1:
        raise ValueError("expert_offsets must have shape [num_experts + 1].")
    if expert_offsets.device != a_cat.device:
        raise ValueError("expert_offsets must be on the same device as input tensors.")
    if a_cat.dtype not in (torch.bfloat16, torch.float16):
        raise ValueError("a_cat dtype must be bf16/fp16.")
    if b_expert.dtype != a_cat.dtype:
        raise ValueError("b_expert dtype should match a_cat dtype.")
    assert expert_offsets.dim() == 1
    if use_atomic_queue and work_counter is not None:
        if work_counter.numel() != 1 or work_counter.dtype != torch.int32:
            raise ValueError("work_counter must be int32 tensor of shape [1].")
        work_counter = work_counter.to(a_cat.device)
    return grouped_gemm(
        a_cat,
        b_expert,
        expert_offsets,
        num_sms=num_sms,
        use_atomic_queue=use_atomic_queue,
        work_counter=work_counter,
    )


def expert_offsets_from_recv_counts(
    num_recv_tokens_per_expert: Union[torch.Tensor, List[int]],
    device: Optional[torch.device] = None,
    dtype: torch.dtype = torch.int32,
) -> torch.Tensor:
    """``[0, c0, c0+c1, ...]`` of length E+1 from per-expert token counts.

    Same contract as src/triton_grouped_gemm.py:300-323: counts are taken as
    int32, summed in 64-bit, and the result cast to ``dtype``.  Device-resident
    counts are summed by a CUDA kernel; counts that stay on the host (a list or
    CPU tensor with no ``device``) are summed by the library's host routine and
    returned on the CPU, as the reference does.
    """
    if isinstance(num_recv_tokens_per_expert, list):
        t = torch.tensor(num_recv_tokens_per_expert, dtype=torch.int32)
    else:
        t = num_recv_tokens_per_expert.flatten()
        if t.dtype not in (torch.int32, torch.int64):
            t = t.to(torch.int32)
    if device is not None:
        t = t.to(device)
    t = t.contiguous()
    out_dtype = dtype if dtype in (torch.int32, torch.int64) else torch.int64
    out = torch.empty(t.numel() + 1, dtype=out_dtype, device=t.device)
    lib = _lib.load()
    counts64 = 1 if t.dtype == torch.int64 else 0
    out64 = 1 if out_dtype == torch.int64 else 0
    if t.device.type == "cuda":
        rc = lib.moe_expert_offsets(
            t.data_ptr(), counts64, t.numel(), out.data_ptr(), out64, _lib.stream_handle(t.device)
        )
        _lib.check_call(rc, "moe_expert_offsets")
    else:
        rc = lib.moe_expert_offsets_host(t.data_ptr(), counts64, t.numel(), out.data_ptr(), out64)
        _lib.check_call(rc, "moe_expert_offsets_host")
    return out if out_dtype == dtype else out.to(dtype)


def reference_grouped_gemm(
    a_cat: torch.Tensor, b_expert: torch.Tensor, expert_offsets: torch.Tensor
) -> torch.Tensor:
    """The reference's per-expert torch loop (src/triton_grouped_gemm.py:446-457).

    Kept as part of the drop-in surface (callers use it as their correctness
    baseline); it is plain torch on whatever device the inputs are on, and rows
    outside every expert segment are left uninitialised, as in the reference.
    """
    out = torch.empty((a_cat.size(0), b_expert.size(2)), device=a_cat.device, dtype=a_cat.dtype)
    bounds = [int(v) for v in expert_offsets.tolist()]
    for e in range(b_expert.size(0)):
        s, t = bounds[e], bounds[e + 1]
        if t > s:
            out[s:t] = a_cat[s:t] @ b_expert[e]
    return out


def tile_list(
    expert_offsets: torch.Tensor,
    m_total: int,
    n_size: int,
    block_m: int = 128,
    block_n: int = 128,
    order: int = 0,
) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
    """Device-decoded (expert, tile_m, tile_n) list, the GEMM scheduler's view.

    ``order=0`` reproduces the list of the reference's ``_build_work_queue``
    (src/triton_grouped_gemm.py:240-297); ``order=1`` is the order the GEMM
    kernel walks.  Returns three int32 CUDA tensors.
    """
    device = expert_offsets.device
    _require_on_device(device)
    offs64 = 1 if expert_offsets.dtype == torch.int64 else 0
    offs = expert_offsets if expert_offsets.dtype in (torch.int32, torch.int64) else expert_offsets.to(torch.int32)
    offs = offs.contiguous()
    num_experts = offs.numel() - 1
    lib = _lib.load()
    count = torch.zeros(1, dtype=torch.int32, device=device)
    stream = _lib.stream_handle(device)
    with torch.cuda.device(device):
        rc = lib.moe_tile_list(offs.data_ptr(), offs64, num_experts, m_total, n_size, block_m,
                               block_n, order, None, None, None, 0, count.data_ptr(), None, stream)
    _lib.check_call(rc, "moe_tile_list")
    total = int(count.item())
    we = torch.empty(total, dtype=torch.int32, device=device)
    wm = torch.empty_like(we)
    wn = torch.empty_like(we)
    if total:
        with torch.cuda.device(device):
            rc = lib.moe_tile_list(offs.data_ptr(), offs64, num_experts, m_total, n_size, block_m,
                                   block_n, order, we.data_ptr(), wm.data_ptr(), wn.data_ptr(),
                                   total, count.data_ptr(), None, stream)
        _lib.check_call(rc, "moe_tile_list")
    return we, wm, wn


def grouped_gemm_wgrad(a: torch.Tensor, b: torch.Tensor, expert_offsets: torch.Tensor, *,
                       out: Optional[torch.Tensor] = None,
                       num_sms: Optional[int] = None) -> torch.Tensor:
    """``out[e] = a[off[e]:off[e+1]].T @ b[off[e]:off[e+1]]`` (weight gradients).

    ``a`` [R, M] and ``b`` [R, N] share the row index (token rows grouped by
    expert); every segment must start and end on a multiple of 64 rows (the
    exchange's ``expert_alignment=64``).  Returns ``[E, M, N]`` in the input dtype.
    """
    device = a.device
    _require_on_device(device, b=b, expert_offsets=expert_offsets, out=out)
    rows, m = a.shape
    num_experts = expert_offsets.numel() - 1
    n = b.shape[1]
    if b.shape[0] != rows or b.dtype != a.dtype or a.dtype not in _DTYPE_CODE:
        raise ValueError("a [R, M] and b [R, N] must share R and a bf16/fp16 dtype")
    if out is None:
        out = torch.empty((num_experts, m, n), dtype=a.dtype, device=device)
    a_c = a if (a.stride(1) == 1 and a.data_ptr() % 16 == 0 and a.stride(0) % 8 == 0) else a.contiguous()
    b_c = b if (b.stride(1) == 1 and b.data_ptr() % 16 == 0 and b.stride(0) % 8 == 0) else b.contiguous()
    offs64 = 1 if expert_offsets.dtype == torch.int64 else 0
    offs = expert_offsets.contiguous() if expert_offsets.dtype in (torch.int32, torch.int64) \
        else expert_offsets.to(torch.int32).contiguous()
    if num_sms is None:
        num_sms = torch.cuda.get_device_properties(device).multi_processor_count
    lib = _lib.load()
    _lib.check_status(device)
    with torch.cuda.device(device):
        rc = lib.moe_grouped_gemm_wgrad(a_c.data_ptr(), a_c.stride(0), b_c.data_ptr(),
                                        b_c.stride(0), out.data_ptr(), out.stride(1), out.stride(0),
                                        offs.data_ptr(), offs64, rows, m, n, num_experts,
                                        _DTYPE_CODE[a.dtype], int(num_sms),
                                        _lib.status_word(device).data_ptr(),
                                        _lib.stream_handle(device))
    _lib.check_call(rc, "moe_grouped_gemm_wgrad")
    return out
