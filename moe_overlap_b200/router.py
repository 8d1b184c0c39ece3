"""Gate softmax / top-k / renormalisation on this package's router kernels.

``SimpleMoE`` routes with ``F.softmax(router(x))`` then ``torch.topk``
(src/train_moe_baseline.py:316-318); the BASELINE configs add a gate bias
(config 5) or renormalise the top-k weights (config 4).  The gate's linear layer
stays a torch matmul (one cuBLAS call, bf16 output as under the reference's
autocast); everything after it is one kernel (``moe_router_topk``), and its
backward another (``moe_router_topk_backward``).
"""
from __future__ import annotations

from typing import Optional

import torch

from . import _lib

__all__ = ["router_topk", "RouterTopK"]


def _launch_fwd(logits: torch.Tensor, bias: Optional[torch.Tensor], top_k: int, renormalize: bool):
    t, e = logits.shape
    dev = logits.device
    if logits.dtype == torch.bfloat16:
        code = _lib.MOE_DTYPE_BF16
    elif logits.dtype == torch.float32:
        code = _lib.MOE_DTYPE_F32
    else:
        raise ValueError("router logits must be bf16 or fp32")
    lg = logits.contiguous()
    b = None
    if bias is not None:
        b = bias.to(device=dev, dtype=torch.float32).contiguous()
        if b.shape != (e,):
            raise ValueError(f"router bias must be [{e}]")
    probs = torch.empty(t, e, dtype=torch.float32, device=dev)
    idx = torch.empty(t, top_k, dtype=torch.int64, device=dev)
    w = torch.empty(t, top_k, dtype=torch.float32, device=dev)
    lib = _lib.load()
    rc = lib.moe_router_topk(lg.data_ptr(), code, b.data_ptr() if b is not None else None, t, e,
                             int(top_k), 1 if renormalize else 0, probs.data_ptr(), idx.data_ptr(),
                             w.data_ptr(), _lib.stream_handle(dev))
    _lib.check_call(rc, "moe_router_topk")
    return probs, idx, w


class RouterTopK(torch.autograd.Function):
    """logits [T, E] (+ bias) -> (probs [T, E], topk_w [T, k]); topk_idx is not differentiable."""

    @staticmethod
    def forward(ctx, logits, bias, top_k, renormalize):
        probs, idx, w = _launch_fwd(logits, bias, top_k, renormalize)
        ctx.save_for_backward(probs, idx)
        ctx.renormalize = renormalize
        ctx.logits_dtype = logits.dtype
        ctx.has_bias = bias is not None
        ctx.mark_non_differentiable(idx)
        ctx.set_materialize_grads(False)  # unused outputs get None, not zero tensors
        return probs, w, idx

    @staticmethod
    def backward(ctx, grad_probs, grad_w, _grad_idx):
        probs, idx = ctx.saved_tensors
        t, e = probs.shape
        k = idx.shape[1]
        if grad_w is None and grad_probs is None:
            return None, None, None, None
        if grad_w is None:
            grad_w = torch.zeros(t, k, dtype=torch.float32, device=probs.device)
        dlogits = torch.empty(t, e, dtype=torch.float32, device=probs.device)
        gw = grad_w.to(torch.float32).contiguous()
        lib = _lib.load()
        rc = lib.moe_router_topk_backward(probs.data_ptr(), idx.data_ptr(), gw.data_ptr(), t, e, k,
                                          1 if ctx.renormalize else 0, dlogits.data_ptr(),
                                          _lib.stream_handle(probs.device))
        _lib.check_call(rc, "moe_router_topk_backward")
        if grad_probs is not None:
            gp = grad_probs.to(torch.float32)
            dlogits = dlogits + probs * (gp - (probs * gp).sum(dim=-1, keepdim=True))
        dbias = dlogits.sum(dim=0) if ctx.has_bias and ctx.needs_input_grad[1] else None
        return dlogits.to(ctx.logits_dtype), dbias, None, None


def router_topk(logits: torch.Tensor, top_k: int, *, bias: Optional[torch.Tensor] = None,
                renormalize: bool = False):
    """(probs [T, E] fp32, topk_idx [T, k] int64, topk_w [T, k] fp32) of the gate logits.

    Differentiable in ``logits`` (and ``bias``) through ``topk_w`` and ``probs``.
    """
    if logits.dim() != 2 or not logits.is_cuda:
        raise ValueError("router logits must be a CUDA tensor [num_tokens, num_experts]")
    probs, w, idx = RouterTopK.apply(logits, bias, int(top_k), bool(renormalize))
    return probs, idx, w
