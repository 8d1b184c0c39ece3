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
