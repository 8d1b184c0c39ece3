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

from .grouped_gemm import gelu_erf, gelu_erf_grad
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
    scale against which rounding differences of the summed terms are measured.

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


def layer_backward_f32(x, router_w, w1, w2, top_k, dout, router_b=None, renormalize=False):
    """Gradients of the routed layer (fp32 math, float64 accumulation).

    Analytic backward of layer_forward_f32: per (token, slot) with expert e,
    a = x W1[e]^T, h = gelu(a), y = h W2[e]^T, out = sum_j w_j y_j; then
    dy = w dout, dw_j = <dout, y_j>, dh = dy W2[e], da = dh * gelu'(a),
    dx += da W1[e], dW2[e] += dy^T h, dW1[e] += da^T x; the top-k weights'
    gradient flows through the optional renormalisation and the softmax into
    the router: dlogits = p * (dp - <p, dp>), dWr = dlogits^T x, dx += dlogits Wr.
    Returns (dx, d_router_w, d_w1, d_w2).
    """
    x64 = x.astype(np.float64)
    probs, idx, w = route(x, router_w, top_k, router_b, renormalize)
    t_count = x.shape[0]
    dx = np.zeros_like(x64)
    dw1 = np.zeros(w1.shape, dtype=np.float64)
    dw2 = np.zeros(w2.shape, dtype=np.float64)
    dwt = np.zeros((t_count, top_k), dtype=np.float64)
    d = dout.astype(np.float64)
    for j in range(top_k):
        for e in np.unique(idx[:, j]):
            rows = np.nonzero(idx[:, j] == e)[0]
            a = x64[rows] @ w1[e].T.astype(np.float64)
            h = gelu_erf(a)
            y = h @ w2[e].T.astype(np.float64)
            dwt[rows, j] = (d[rows] * y).sum(axis=1)
            dy = w[rows, j:j + 1].astype(np.float64) * d[rows]
            dh = dy @ w2[e].astype(np.float64)
            da = dh * gelu_erf_grad(a)
            dx[rows] += da @ w1[e].astype(np.float64)
            dw2[e] += dy.T @ h
            dw1[e] += da.T @ x64[rows]
    if renormalize:
        raw = np.take_along_axis(probs, idx, axis=-1).astype(np.float64)
        ssum = raw.sum(axis=-1, keepdims=True)
        wt = raw / ssum
        dwt = (dwt - (dwt * wt).sum(axis=-1, keepdims=True)) / ssum
    dp = np.zeros(probs.shape, dtype=np.float64)
    np.put_along_axis(dp, idx, dwt, axis=-1)
    p64 = probs.astype(np.float64)
    dlogits = p64 * (dp - (p64 * dp).sum(axis=-1, keepdims=True))
    d_router = dlogits.T @ x64
    dx += dlogits @ router_w.astype(np.float64)
    return dx, d_router, dw1, dw2


def experts_backward_bf16(x_bits, idx, w, w1_bits, w2_bits, dout_bits):
    """Routed-expert gradients at the build's rounding points, for a given routing.

    Per (token, slot) with expert e (numpy fp32 matmuls, bf16 where the pipeline
    stores):  a = x W1[e]^T (fp32), g = bf16(gelu'(a)), h = bf16(gelu(a)), y = bf16(h W2[e]^T);
    dy = bf16(w * dout); dpre = bf16((dy W2[e]) * g); dxr = bf16(dpre W1[e]).
    Returns a dict of
      ``dx``   bf16 bits [T, H]: the slot sum of dxr in fp32, rounded once;
      ``dw``   float64 [T, k]:  <dout, y>;
      ``dw1``  bf16 bits [E, F, H] = sum dpre^T x;  ``dw2`` bf16 bits [E, H, F] = sum dy^T h;
      ``mag_dx``, ``mag_dw1``, ``mag_dw2``: the sums of absolute terms behind each
      element, against which summation-order differences are measured.
    """
    t_count, hidden = x_bits.shape
    n_exp, ffn, _ = w1_bits.shape
    rnd = lambda v: bf16_bits_to_f32(f32_to_bf16_bits(np.asarray(v, dtype=np.float32)))
    xf, dof = bf16_bits_to_f32(x_bits), bf16_bits_to_f32(dout_bits)
    dx = np.zeros((t_count, hidden), np.float32)
    mag_dx = np.zeros_like(dx)
    dw = np.zeros(idx.shape, np.float64)
    dw1 = np.zeros((n_exp, ffn, hidden), np.float32)
    dw2 = np.zeros((n_exp, hidden, ffn), np.float32)
    mag1, mag2 = np.zeros_like(dw1), np.zeros_like(dw2)
    for e in range(n_exp):
        sel = np.argwhere(idx == e)
        if sel.size == 0:
            continue
        toks, slots = sel[:, 0], sel[:, 1]
        w1f, w2f = bf16_bits_to_f32(w1_bits[e]), bf16_bits_to_f32(w2_bits[e])
        acc = xf[toks] @ w1f.T
        gsave = rnd(gelu_erf_grad(acc))
        h = rnd(gelu_erf(acc))
        y = rnd(h @ w2f.T)
        dw[toks, slots] = (dof[toks].astype(np.float64) * y).sum(axis=1)
        dy = rnd(w[toks, slots][:, None].astype(np.float32) * dof[toks])
        dpre = rnd((dy @ w2f) * gsave)
        dxr = rnd(dpre @ w1f)
        np.add.at(dx, toks, dxr)
        np.add.at(mag_dx, toks, np.abs(dxr))
        dw2[e] = dy.T @ h
        dw1[e] = dpre.T @ xf[toks]
        mag2[e] = np.abs(dy).T @ np.abs(h)
        mag1[e] = np.abs(dpre).T @ np.abs(xf[toks])
    return dict(dx=f32_to_bf16_bits(dx), dw=dw, dw1=f32_to_bf16_bits(dw1),
                dw2=f32_to_bf16_bits(dw2), mag_dx=mag_dx, mag_dw1=mag1, mag_dw2=mag2)


def topk_from_logits(logits, top_k: int, router_b=None, renormalize: bool = False):
    """(probs, topk_idx, topk_w) of given logits [T, E] (fp32 arithmetic, ties to the
    lower expert id): the steps after the gate's linear layer in route()."""
    z = np.asarray(logits, np.float32)
    if router_b is not None:
        z = z + np.asarray(router_b, np.float32)
    probs = softmax(z).astype(np.float32)
    idx = np.argsort(-probs, axis=-1, kind="stable")[:, :top_k].astype(np.int64)
    w = np.take_along_axis(probs, idx, axis=-1)
    if renormalize:
        w = w / w.sum(axis=-1, keepdims=True)
    return probs, idx, w.astype(np.float32)


def topk_backward(probs, idx, dw, renormalize: bool = False):
    """d loss / d logits for the upstream gradient dw [T, k] of topk_from_logits'
    weights (float64): through the renormalisation, scattered to the selected
    experts, then the softmax backward p * (dp - <p, dp>)."""
    p = np.asarray(probs, np.float64)
    d = np.asarray(dw, np.float64)
    sel = np.take_along_axis(p, idx, axis=-1)
    if renormalize:
        s = sel.sum(axis=-1, keepdims=True)
        d = (d - (d * (sel / s)).sum(axis=-1, keepdims=True)) / s
    dp = np.zeros_like(p)
    np.put_along_axis(dp, idx, d, axis=-1)
    return p * (dp - (p * dp).sum(axis=-1, keepdims=True))
