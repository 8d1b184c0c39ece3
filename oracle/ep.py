"""Oracle for the expert-parallel token exchange (test infrastructure only).

Restates in numpy what the reference's dispatch/combine path computes:
  * ``dispatch_layout``: DeepEP's ``get_dispatch_layout``
    (thirdParty/DeepEP/csrc/kernels/layout.cu:10-121, as re-derived in pure
    torch by thirdParty/DeepEP/tests/test_intranode.py:41-66): tokens per
    expert, tokens per rank counted once per token, and ``is_token_in_rank``.
  * ``dispatch``: the data movement of ``DeepEPDispatcher.dispatch``
    (src/deep_ep_comm.py:69-105) in this build's expert-ordered receive layout:
    one row per (token, selected expert) on the rank that owns the expert
    (experts sharded contiguously, E/W per rank, src/train_moe_baseline.py:136-137),
    rows grouped by local expert, then by source rank, then by (token, slot).
    ``recv_topk_idx`` holds the local expert id in the row's slot and -1
    elsewhere, ``recv_topk_weights`` the weight there and 0 elsewhere, the same
    convention DeepEP uses for slots that are not local (intranode.cu:385-394).
  * ``combine``: DeepEP's intranode combine (intranode.cu:961-1030): for each
    original token the fp32 sum of the rows returned for it, rounded once to
    bf16; with ``weights`` it is the fused weighted top-k sum
    ``sum_j w[t, j] * y[row(t, j)]`` that the reference computes as
    ``recv_y += y * gate`` before an unweighted combine
    (src/train_moe_baseline.py:394-399, src/deep_ep_comm.py:107-115).
"""
from __future__ import annotations

import numpy as np

from .numerics import bf16_bits_to_f32, f32_to_bf16_bits


def dispatch_layout(topk_idx: np.ndarray, num_experts: int, world: int):
    """(num_tokens_per_rank [W] int32, num_tokens_per_expert [E] int32, is_token_in_rank [T, W] bool)."""
    idx = np.asarray(topk_idx, dtype=np.int64)
    t = idx.shape[0]
    per_rank = num_experts // world
    valid = (idx >= 0) & (idx < num_experts)
    per_expert = np.bincount(idx[valid], minlength=num_experts).astype(np.int32)
    in_rank = np.zeros((t, world), dtype=bool)
    rows, cols = np.nonzero(valid)
    in_rank[rows, idx[rows, cols] // per_rank] = True
    per_rank_counts = in_rank.sum(axis=0).astype(np.int32)
    return per_rank_counts, per_expert, in_rank


def dispatch(xs, topk_idxs, topk_weights, num_experts: int, expert_alignment: int = 1,
             scale_rows: bool = False):
    """Expert-ordered dispatch over ``W = len(xs)`` ranks.

    ``expert_alignment`` rounds each local expert's segment up to a multiple of
    that many rows (DeepEP's dispatch argument of that name,
    thirdParty/DeepEP/deep_ep/buffer.py:327); the padding rows are zero with
    ``topk_idx`` -1, weight 0 and source (-1, -1).

    xs[r]: [T_r, H] bf16 bits (uint16); topk_idxs[r]: [T_r, k] int64 global
    expert ids (-1 = none); topk_weights[r]: [T_r, k] float32.
    Returns (recv, send_pos) where recv[d] is a dict with ``x`` [n, H],
    ``topk_idx`` [n, k], ``topk_weights`` [n, k], ``src_rank`` [n], ``src_token``
    [n], ``offsets`` [E/W + 1] int32; and send_pos[r] is [T_r, k] int32, the
    row on the owning rank of every (token, slot) (-1 for none).
    """
    world = len(xs)
    per_rank = num_experts // world
    k = topk_idxs[0].shape[1] if world else 0
    # Assignments per destination, ordered by (local expert, src rank, token, slot).
    buckets = [[[] for _ in range(per_rank)] for _ in range(world)]
    for r in range(world):
        idx = np.asarray(topk_idxs[r], dtype=np.int64)
        for t in range(idx.shape[0]):
            for j in range(k):
                e = int(idx[t, j])
                if 0 <= e < num_experts:
                    buckets[e // per_rank][e % per_rank].append((r, t, j))
    recv, send_pos = [], [np.full(np.asarray(topk_idxs[r]).shape, -1, np.int32) for r in range(world)]
    al = max(1, int(expert_alignment))
    for d in range(world):
        order, counts = [], []
        for le in range(per_rank):
            seg = list(buckets[d][le])
            padded = -(-len(seg) // al) * al
            counts.append(padded)
            order += seg + [None] * (padded - len(seg))
        n = len(order)
        hidden = xs[0].shape[1]
        rx = np.zeros((n, hidden), dtype=np.uint16)
        ridx = np.full((n, k), -1, dtype=np.int64)
        rw = np.zeros((n, k), dtype=np.float32)
        src_rank = np.full(n, -1, dtype=np.int32)
        src_tok = np.full(n, -1, dtype=np.int32)
        for row, item in enumerate(order):
            if item is None:
                continue
            r, t, j = item
            e = int(topk_idxs[r][t, j])
            if scale_rows:
                prod = bf16_bits_to_f32(xs[r][t]) * np.float32(topk_weights[r][t, j])
                rx[row] = f32_to_bf16_bits(prod.astype(np.float32))
            else:
                rx[row] = xs[r][t]
            ridx[row, j] = e % per_rank
            rw[row, j] = topk_weights[r][t, j]
            src_rank[row], src_tok[row] = r, t
            send_pos[r][t, j] = row
        offsets = np.zeros(per_rank + 1, dtype=np.int32)
        offsets[1:] = np.cumsum(counts)
        recv.append(dict(x=rx, topk_idx=ridx, topk_weights=rw, src_rank=src_rank,
                         src_token=src_tok, offsets=offsets))
    return recv, send_pos


def dispatch_fp8(xqs, scales, topk_idxs, topk_weights, num_experts: int):
    """Dispatch of an FP8 payload (DeepEP's (x_fp8, x_scales) pair,
    thirdParty/DeepEP/deep_ep/buffer.py:338-342): the same receive layout and
    metadata as ``dispatch``, with each receive row holding its source token's
    e4m3 bytes and per-128 scales unchanged (intranode.cu:397-402 copies the
    scales next to the row).  ``recv[d]`` gains ``x_fp8`` [n, H] uint8 and
    ``x_scales`` [n, H/128] float32 (zero on rows without a source).
    """
    zeros = [np.zeros((np.asarray(q).shape[0], 1), dtype=np.uint16) for q in xqs]
    recv, send_pos = dispatch(zeros, topk_idxs, topk_weights, num_experts)
    for d in recv:
        n = d["src_rank"].shape[0]
        h = np.asarray(xqs[0]).shape[1]
        d["x_fp8"] = np.zeros((n, h), dtype=np.uint8)
        d["x_scales"] = np.zeros((n, h // 128), dtype=np.float32)
        for row in range(n):
            r, t = int(d["src_rank"][row]), int(d["src_token"][row])
            if r >= 0:
                d["x_fp8"][row] = xqs[r][t]
                d["x_scales"][row] = scales[r][t]
        del d["x"]
    return recv, send_pos


def dispatch_cached(xs, topk_idxs, topk_weights, num_experts: int, src_recv, src_send_pos,
                    scale_rows: bool = False):
    """Cached re-dispatch (DeepEP's dispatch given a handle,
    thirdParty/DeepEP/deep_ep/buffer.py:383-390): new rows ``xs`` for the tokens
    and top-k choices of an earlier dispatch, whose result was (src_recv,
    src_send_pos).  Each (token, slot) row goes to the row that dispatch gave it;
    every receiver keeps that dispatch's metadata and offsets, and its alignment
    padding rows are zero.  Same return shape as ``dispatch``.
    """
    world = len(xs)
    per_rank = num_experts // world
    recv = []
    for d in range(world):
        src = src_recv[d]
        n = int(src["offsets"][-1])
        rx = np.zeros((n, xs[0].shape[1]), dtype=np.uint16)
        recv.append(dict(x=rx, topk_idx=src["topk_idx"].copy(), topk_weights=src["topk_weights"].copy(),
                         src_rank=src["src_rank"].copy(), src_token=src["src_token"].copy(),
                         offsets=src["offsets"].copy()))
    for r in range(world):
        idx = np.asarray(topk_idxs[r], dtype=np.int64)
        for (t, j), row in np.ndenumerate(src_send_pos[r]):
            e = int(idx[t, j])
            if row < 0 or not 0 <= e < num_experts:
                continue
            if scale_rows:
                prod = bf16_bits_to_f32(xs[r][t]) * np.float32(topk_weights[r][t, j])
                recv[e // per_rank]["x"][row] = f32_to_bf16_bits(prod.astype(np.float32))
            else:
                recv[e // per_rank]["x"][row] = xs[r][t]
    return recv, [np.array(s, copy=True) for s in src_send_pos]


def topk_weight_grad(grad_outs, ys, topk_idxs, send_pos, num_experts: int):
    """d loss / d w[t, j] of the weighted combine: <grad_out[t], y_{owner}(row(t, j))>
    in float64 (the product sums in fp32 in its own order), 0 for empty slots."""
    world = len(ys)
    per_rank = num_experts // world
    outs = []
    for r in range(world):
        idx = np.asarray(topk_idxs[r], dtype=np.int64)
        g = bf16_bits_to_f32(grad_outs[r]).astype(np.float64)
        out = np.zeros(idx.shape, dtype=np.float64)
        for (t, j), pos in np.ndenumerate(send_pos[r]):
            if pos >= 0:
                y = bf16_bits_to_f32(ys[int(idx[t, j]) // per_rank][pos]).astype(np.float64)
                out[t, j] = float(g[t] @ y)
        outs.append(out)
    return outs


def combine(ys, topk_idxs, send_pos, num_experts: int, weights=None):
    """Per-source combine.  ys[d]: [n_d, H] bf16 bits of the rows each rank returns.

    out[r][t] = bf16( sum_j s_j * y_{owner(t,j)}[send_pos[r][t, j]] ) with
    s_j = 1 (unweighted, the reference combine) or weights[r][t, j].
    """
    world = len(ys)
    per_rank = num_experts // world
    outs = []
    for r in range(world):
        idx = np.asarray(topk_idxs[r], dtype=np.int64)
        t_count, k = idx.shape
        hidden = ys[0].shape[1] if ys[0].ndim == 2 else 0
        acc = np.zeros((t_count, hidden), dtype=np.float32)
        for j in range(k):
            pos = send_pos[r][:, j]
            for t in np.nonzero(pos >= 0)[0]:
                d = int(idx[t, j]) // per_rank
                row = bf16_bits_to_f32(ys[d][pos[t]])
                s = np.float32(1.0) if weights is None else np.float32(weights[r][t, j])
                acc[t] += s * row
        outs.append(f32_to_bf16_bits(acc))
    return outs
