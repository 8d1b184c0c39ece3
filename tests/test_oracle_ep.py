"""CPU checks of the exchange oracle (oracle/ep.py) on its own properties."""
import numpy as np
import pytest
import torch

from oracle import ep as oep
from tests._inputs import to_storage


def _routing(world, tokens, num_experts, topk, seed, hidden=64):
    g = torch.Generator().manual_seed(seed)
    xs, idxs, ws = [], [], []
    for _ in range(world):
        xs.append(to_storage(torch.randn(tokens, hidden, generator=g).to(torch.bfloat16)))
        idx = torch.topk(torch.rand(tokens, num_experts, generator=g), topk, dim=-1).indices
        idx[torch.rand(tokens, topk, generator=g) < 0.1] = -1
        idxs.append(idx.numpy().astype(np.int64))
        ws.append(torch.rand(tokens, topk, generator=g).numpy().astype(np.float32))
    return xs, idxs, ws


@pytest.mark.parametrize("world,align,scale", [(1, 1, False), (2, 64, True), (4, 16, False),
                                               (4, 1, True)])
def test_cached_dispatch_equals_a_full_dispatch_of_the_new_rows(world, align, scale):
    """Rows placed by an earlier dispatch's positions land exactly where a full
    dispatch of the new rows with the same routing puts them."""
    E, tokens, topk = 8, 50, 2
    xs, idxs, ws = _routing(world, tokens, E, topk, seed=world * 10 + align)
    x2 = [((x.astype(np.int32) + 7) & 0x7FFF).astype(np.uint16) for x in xs]  # other finite rows
    src_recv, src_pos = oep.dispatch(xs, idxs, ws, E, expert_alignment=align)
    got, got_pos = oep.dispatch_cached(x2, idxs, ws, E, src_recv, src_pos, scale_rows=scale)
    want, want_pos = oep.dispatch(x2, idxs, ws, E, expert_alignment=align, scale_rows=scale)
    for d in range(world):
        for key in want[d]:
            assert np.array_equal(got[d][key], want[d][key]), (d, key)
    for r in range(world):
        assert np.array_equal(got_pos[r], want_pos[r])


@pytest.mark.parametrize("world,topk,num_experts", [(1, 2, 8), (2, 2, 16), (4, 3, 16), (8, 2, 16)])
def test_oracle_dispatch_combine_satisfy_deepep_test_invariants(world, topk, num_experts):
    """The exchange oracle against the invariants DeepEP's own intranode test asserts
    (thirdParty/DeepEP/tests/test_intranode.py:119-131 counts and local ids, :80-86
    rows tagged by source, :168-183 combine / #hits == x), restated for rows that are
    one per (token, local expert).  Token rows carry their (rank, token) tag in
    column 0, as src/verify_deepep_dispatch.py:62-64 does (rank*32+token here, exact
    in bf16 for up to 8 ranks of 32 tokens)."""
    from oracle.numerics import bf16_bits_to_f32, f32_to_bf16_bits

    tokens, hidden = 32, 16
    g = np.random.default_rng(world * 10 + topk)
    xs, idxs, ws = [], [], []
    for r in range(world):
        xf = np.zeros((tokens, hidden), np.float32)
        xf[:, 0] = r * tokens + np.arange(tokens)
        xf[:, 1:] = g.integers(-4, 5, size=(tokens, hidden - 1))
        xs.append(f32_to_bf16_bits(xf))
        idx = np.stack([g.permutation(num_experts)[:topk] for _ in range(tokens)]).astype(np.int64)
        idx[g.random((tokens, topk)) < 0.1] = -1
        idxs.append(idx)
        ws.append(g.random((tokens, topk)).astype(np.float32))
    recv, send_pos = oep.dispatch(xs, idxs, ws, num_experts)
    per_rank = num_experts // world
    glob = np.bincount(np.concatenate([i[i >= 0] for i in idxs]), minlength=num_experts)
    for d in range(world):
        r = recv[d]
        n = int(r["offsets"][-1])
        assert n == int(glob[d * per_rank:(d + 1) * per_rank].sum())       # rows received
        assert np.diff(r["offsets"]).tolist() == glob[d * per_rank:(d + 1) * per_rank].tolist()
        ids = r["topk_idx"][:n]
        assert np.all((ids == -1) | ((ids >= 0) & (ids < per_rank)))
        assert np.all((ids >= 0).sum(axis=1) == 1)                         # one slot per row
        for le in range(per_rank):
            assert int((ids == le).sum()) == int(glob[d * per_rank + le])
            seg = slice(r["offsets"][le], r["offsets"][le + 1])
            assert np.all(np.diff(r["src_rank"][seg]) >= 0)                # source-rank order
        tag = bf16_bits_to_f32(r["x"][:n, 0])
        assert np.array_equal(tag, (r["src_rank"][:n] * tokens + r["src_token"][:n]).astype(np.float32))
        for row in range(n):                                                # the token's own row
            assert np.array_equal(r["x"][row, 1:], xs[r["src_rank"][row]][r["src_token"][row], 1:])
    # combine of identity expert outputs, unweighted: x times the token's number of hits
    ys = [recv[d]["x"][: int(recv[d]["offsets"][-1])] for d in range(world)]
    outs = oep.combine(ys, idxs, send_pos, num_experts)
    for r in range(world):
        hits = (idxs[r] >= 0).sum(axis=1).astype(np.float32)[:, None]
        # the sum starts from +0, so a token with no hits gets +0, never -0
        want = f32_to_bf16_bits(np.float32(0.0) + bf16_bits_to_f32(xs[r])[:, 1:] * hits)
        assert np.array_equal(outs[r][:, 1:], want)
