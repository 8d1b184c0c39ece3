"""Oracle for the routed MoE layer (test infrastructure only).

Restates SimpleMoE's routed path (src/train_moe_baseline.py):
  * router: linear without bias (:141) -> softmax (:317) -> top-k without
    renormalisation (:318); the BASELINE configs add a gate bias (config 5) or
    renormalise the top-k weights (config 4), applied here the same way to both
    sides when asked;
  * experts: ExpertMLP w2(gelu(w1(x))) with exact (erf) GELU and no biases (:86-93);
  * output: sum over slots of gate * expert(x) (:343-348);
  * router stats: per-expert assignment counts, entropy, std, cv (:450-461).
``layer_forward_bf16`` follows the rounding points of this build's pipeline
(bf16 weights/activations, fp32 accumulation, GELU on the fp32 accumulator,
bf16 hidden and expert outputs, fp32 weighted sum rounded once) so that GPU
results can be compared tightly.
"""
from __future__ import annotations

import numpy as np

from .grouped_gemm import gelu_erf
from .numerics import bf16_bits_to_f32, f32_to_bf16_bits


def softmax(logits: np.ndarray) -> np.ndarray:
    z = logits - logits.max(axis=-1, keepdims=True)
    e = np.exp(z)
    return e / e.sum(axis=-1, keepdims=True)


def route(x: np.ndarray, router_w: np.ndarray, top_k: int, router_b=None,
          renormalize: bool = False, bf16_logits: bool = False):
    """(probs [T, E], topk_idx [T, k] int64, topk_w [T, k] float32), float32 arithmetic.

    ``bf16_logits`` rounds the router's linear output to bf16 before the fp32
    softmax, which is what the reference's bf16 autocast run does
    (src/train_moe_baseline.py:548-550: nn.Linear under autocast returns bf16,
    F.softmax is computed in fp32).
    """
    logits = x.astype(np.float32) @ router_w.astype(np.float32).T
    if bf16_logits:
        logits = bf16_bits_to_f32(f32_to_bf16_bits(logits.astype(np.float32)))
    if router_b is not None:
        logits = logits + router_b.astype(np.float32)
    probs = softmax(logits.astype(np.float32)).astype(np.float32)
    idx = np.argsort(-probs, axis=-1, kind="stable")[:, :top_k].astype(np.int64)
    w = np.take_along_axis(probs, idx, axis=-1)
    if renormalize:
        w = w / w.sum(axis=-1, keepdims=True)
    return probs, idx, w.astype(np.float32)


def layer_forward_f32(x, router_w, w1, w2, top_k, router_b=None, renormalize=False):
    """fp32 SimpleMoE routed forward; w1 [E, F, H], w2 [E, H, F] (nn.Linear layout)."""
    _, idx, w = route(x, router_w, top_k, router_b, renormalize)
    out = np.zeros_like(x, dtype=np.float32)
    for j in range(top_k):
        for e in np.unique(idx[:, j]):
            rows = np.nonzero(idx[:, j] == e)[0]
            h = gelu_erf(x[rows].astype(np.float32) @ w1[e].T).astype(np.float32)
            y = h @ w2[e].T
            out[rows] += w[rows, j:j + 1] * y
    return out


def layer_forward_bf16(x_bits, idx, w, w1_bits, w2_bits, expert_offset: int = 0,
                       return_magnitude: bool = False):
    """The build's rounding points, for a given routing; returns bf16 bits [T, H].

    With ``return_magnitude`` also returns sum_j |w_j * y_j| per element, the
    scale against which rounding differences of the summed terms are judged.

    x_bits [T, H], w1_bits [E_local, F, H], w2_bits [E_local, H, F] are bf16 bit
    patterns; idx holds global expert ids (experts outside
    [expert_offset, expert_offset + E_local) contribute nothing).
    """
    t_count, hidden = x_bits.shape
    n_local = w1_bits.shape[0]
    xf = bf16_bits_to_f32(x_bits)
    y_rows = {}
    for e in range(n_local):
        sel = np.argwhere(idx == expert_offset + e)
        if sel.size == 0:
            continue
        toks = sel[:, 0]
        acc = xf[toks] @ bf16_bits_to_f32(w1_bits[e]).T
        h = bf16_bits_to_f32(f32_to_bf16_bits(gelu_erf(acc).astype(np.float32)))
        y = bf16_bits_to_f32(f32_to_bf16_bits(h @ bf16_bits_to_f32(w2_bits[e]).T))
        for (t, j), row in zip(sel, y):
            y_rows[(int(t), int(j))] = row
    out = np.zeros((t_count, hidden), dtype=np.float32)
    mag = np.zeros((t_count, hidden), dtype=np.float32)
    for j in range(idx.shape[1]):
        for t in range(t_count):
            row = y_rows.get((t, j))
            if row is not None:
                term = np.float32(w[t, j]) * row
                out[t] = out[t] + term
                mag[t] += np.abs(term)
    if return_magnitude:
        return f32_to_bf16_bits(out), mag
    return f32_to_bf16_bits(out)


def router_stats(probs: np.ndarray, idx: np.ndarray, num_experts: int):
    """(entropy, load_std, load_cv) as src/train_moe_baseline.py:450-461 computes them."""
    counts = np.bincount(idx.reshape(-1), minlength=num_experts).astype(np.float64)
    mean = max(counts.mean(), 1e-6)
    entropy = float((-probs * np.log(np.maximum(probs, 1e-9))).sum(axis=-1).mean())
    std = float(counts.std(ddof=1))
    return entropy, std, std / mean
