"""GPU checks of the tile-granular dispatch/GEMM overlap (expert-ordered dispatch).

The expert-ordered dispatch must place every row exactly as the oracle's
dispatch does (rows, local ids, weights, source tags, offsets, send positions:
bit-exact), count every row it delivers in the owner's per-expert arrival
counters, and ``moe_ep_expert_gemm`` (the up-projection that waits per expert
for those counters) must give the grouped GEMM's result bit for bit.  W ranks
are emulated on one GPU by LocalGroup, each phase run for all ranks before the
next, so every wait finds its counters already complete.  A wait that nothing
satisfies must expire with MOE_ERR_TIMEOUT and leave the context usable, and
the layer with the overlap must reproduce the layer without it bit for bit.
"""
import numpy as np
import pytest
import torch

import moe_overlap_b200 as mo
from moe_overlap_b200 import _lib
from moe_overlap_b200.ep import LocalGroup
from oracle import ep as oep
from tests._inputs import to_storage

pytestmark = pytest.mark.gpu


def _routing(world, tokens, num_experts, topk, seed, hidden):
    g = torch.Generator().manual_seed(seed)
    xs, idxs, ws = [], [], []
    for _ in range(world):
        xs.append(torch.randn(tokens, hidden, generator=g).to(torch.bfloat16))
        idx = torch.topk(torch.rand(tokens, num_experts, generator=g), topk).indices.to(torch.int64)
        idx[torch.rand(tokens, topk, generator=g) < 0.05] = -1
        idxs.append(idx)
        ws.append(torch.rand(tokens, topk, generator=g))
    return xs, idxs, ws


@pytest.mark.parametrize("world,tokens,topk,num_experts", [(1, 700, 2, 16), (2, 513, 2, 16),
                                                           (4, 300, 3, 16), (8, 200, 2, 16)])
def test_ordered_dispatch_and_expert_gemm_match(cuda_device, world, tokens, topk, num_experts):
    hidden, n = 256, 384
    xs, idxs, ws = _routing(world, tokens, num_experts, topk, world * 7 + topk, hidden)
    cap = world * tokens * topk
    grp = LocalGroup(world, num_experts, hidden, tokens, topk, cap, num_blocks=9)
    recv, send_pos = oep.dispatch([to_storage(x) for x in xs], [i.numpy() for i in idxs],
                                  [w.numpy() for w in ws], num_experts)
    g = torch.Generator().manual_seed(5)
    per_rank = num_experts // world
    b = (torch.randn(per_rank, hidden, n, generator=g) * 0.05).to(torch.bfloat16).to(cuda_device)
    try:
        dx = [x.to(cuda_device) for x in xs]
        di = [i.to(cuda_device) for i in idxs]
        dw = [w.to(cuda_device) for w in ws]
        slot, _ = grp.dispatch_ordered(dx, di, dw, pad_rows=True)
        torch.cuda.synchronize()
        assert int(grp.status.item()) == 0, _lib.status_string(int(grp.status.item()))
        for d, ep in enumerate(grp.eps):
            v, want = ep.slots[slot], recv[d]
            n_rows = int(want["offsets"][-1])
            assert np.array_equal(v.expert_offsets.cpu().numpy(), want["offsets"])
            assert np.array_equal(to_storage(v.recv_x[:n_rows]), want["x"])
            assert np.array_equal(v.recv_topk_idx[:n_rows, :topk].cpu().numpy(), want["topk_idx"])
            assert np.array_equal(v.recv_topk_weights[:n_rows, :topk].cpu().numpy(), want["topk_weights"])
            src = v.recv_src[:n_rows].cpu().numpy()
            assert np.array_equal(src[:, 0], want["src_rank"]) and np.array_equal(src[:, 1], want["src_token"])
            counts = np.diff(want["offsets"])
            # every row was counted on arrival, and the expected counts are the segment sizes
            assert np.array_equal(v.arrived.cpu().numpy(), counts.astype(np.int32))
            assert np.array_equal(v.expected.cpu().numpy(), counts.astype(np.int32))
        for r, ep in enumerate(grp.eps):
            t, k = idxs[r].shape
            assert np.array_equal(ep.slots[slot].send_pos[:t * k].cpu().numpy().reshape(t, k), send_pos[r])
        for act in (None, "gelu"):
            for ep in grp.eps:
                out = torch.full((cap, n), 3.0, dtype=torch.bfloat16, device=cuda_device)
                ctr = torch.zeros(1, dtype=torch.int32, device=cuda_device)
                ep.expert_gemm(slot, b, out, act, 148, True, ctr, grp.wait_ns, grp.status)
                v = ep.slots[slot]
                want = mo.grouped_gemm(v.recv_x, b, v.expert_offsets, activation=act)
                torch.cuda.synchronize()
                assert int(grp.status.item()) == 0
                rows = int(v.expert_offsets[-1])
                assert torch.equal(out[:rows], want[:rows])
                assert bool((out[rows:] == 3.0).all())  # rows past the received count untouched
        # the combine of an ordered dispatch is the ordinary one
        outs = [torch.empty(tokens, hidden, dtype=torch.bfloat16, device=cuda_device) for _ in range(world)]
        ys = []
        for ep in grp.eps:
            rows = int(ep.slots[slot].expert_offsets[-1])
            y = (ep.slots[slot].recv_x[:rows].float() * 0.5).to(torch.bfloat16)
            ep.slots[slot].expert_out[:rows].copy_(y)
            ys.append(to_storage(y))
        grp.combine(di, dw, slot, grp.epoch, False, outs)
        torch.cuda.synchronize()
        want_c = oep.combine(ys, [i.numpy() for i in idxs], send_pos, num_experts)
        for r in range(world):
            assert np.array_equal(to_storage(outs[r]), want_c[r])
    finally:
        grp.close()


def test_expert_gemm_wait_that_nobody_satisfies_times_out(cuda_device, monkeypatch):
    """An arrival counter that nothing raises: the GEMM gives up after its bound, records
    MOE_ERR_TIMEOUT and the context stays usable."""
    world, tokens, topk, num_experts, hidden = 2, 256, 2, 8, 128
    xs, idxs, ws = _routing(world, tokens, num_experts, topk, 3, hidden)
    grp = LocalGroup(world, num_experts, hidden, tokens, topk, world * tokens * topk, num_blocks=4)
    try:
        slot, _ = grp.dispatch_ordered([x.to(cuda_device) for x in xs], [i.to(cuda_device) for i in idxs],
                                       [w.to(cuda_device) for w in ws])
        torch.cuda.synchronize()
        assert int(grp.status.item()) == 0
        ep = grp.eps[0]
        v = ep.slots[slot]
        assert int(v.expected.sum()) > 0
        v.arrived.zero_()  # as if no peer had delivered anything
        b = torch.randn(num_experts // world, hidden, 128, device=cuda_device).to(torch.bfloat16)
        out = torch.empty(world * tokens * topk, 128, dtype=torch.bfloat16, device=cuda_device)
        status = torch.zeros(1, dtype=torch.int32, device=cuda_device)
        ep.expert_gemm(slot, b, out, None, 8, True, torch.zeros(1, dtype=torch.int32, device=cuda_device),
                       50_000_000, status)  # 50 ms bound
        torch.cuda.synchronize()
        assert int(status.item()) == _lib.MOE_ERR_TIMEOUT
        # the context still works
        c = mo.grouped_gemm(v.recv_x, b, v.expert_offsets)
        torch.cuda.synchronize()
        assert c.shape[1] == 128
    finally:
        grp.close()


def test_ordered_scatter_requires_the_slots_ordered_begin(cuda_device):
    """The ordered scatter sends the order its begin built: after a plain begin on the
    slot, or with another token count, it is refused on the host before any launch."""
    world, tokens, topk, num_experts, hidden = 1, 128, 2, 8, 128
    xs, idxs, ws = _routing(world, tokens, num_experts, topk, 4, hidden)
    grp = LocalGroup(world, num_experts, hidden, tokens, topk, tokens * topk, num_blocks=4)
    try:
        ep = grp.eps[0]
        x, i, w = xs[0].to(cuda_device), idxs[0].to(cuda_device), ws[0].to(cuda_device)
        status = torch.zeros(1, dtype=torch.int32, device=cuda_device)
        ep.dispatch_begin(x, i, w, 0, 1, status)
        with pytest.raises(_lib.MoeError):
            ep.dispatch_ordered_scatter(x, i, w, 0, 1, 4, False, grp.wait_ns, status)
        ep.dispatch_ordered_begin(x, i, w, 1, 1, status)
        with pytest.raises(_lib.MoeError):
            ep.dispatch_ordered_scatter(x[:64], i[:64], w[:64], 1, 1, 4, False, grp.wait_ns, status)
        torch.cuda.synchronize()
        assert int(status.item()) == 0
    finally:
        grp.close()


def test_layer_with_tile_overlap_equals_layer_without(cuda_device):
    from moe_overlap_b200.layer import MoELayer

    tokens, hidden, ffn, experts, topk = 1536, 256, 512, 8, 2
    g = torch.Generator().manual_seed(41)
    x = torch.randn(tokens, hidden, generator=g).to(torch.bfloat16).to(cuda_device)
    base = MoELayer(hidden, ffn, experts, topk, micro_batch_size=512, num_comm_sms=8).init_random(0.05, 6)
    over = MoELayer(hidden, ffn, experts, topk, micro_batch_size=512, num_comm_sms=8,
                    overlap_tiles=True).init_random(0.05, 6)
    try:
        routing = base.route(x)
        want, _ = base(x, routing=routing)
        for _ in range(2):  # both slots
            got, _ = over(x, routing=routing)
            torch.cuda.synchronize()
            assert torch.equal(got, want)
        mo.check_status(cuda_device, sync=True)
    finally:
        base.close()
        over.close()
