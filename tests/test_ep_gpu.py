"""GPU parity of the expert-parallel exchange against the CPU oracle (oracle/ep.py).

W ranks are emulated on one GPU by LocalGroup (every rank's endpoint in this
process, each phase run for all ranks before the next), so the peer stores,
flags and pulls are the same code the multi-GPU path runs.  Everything the
exchange moves is compared bit for bit: received rows (bf16 copies), local
expert ids, weights, source tags, expert_offsets and send positions; the
combine sums in fp32 in slot order exactly as the oracle does, so it is
bit-exact too.  The DeepEP test invariants (thirdParty/DeepEP/tests/
test_intranode.py:62-66 layout, :119-131 counts and local ids) are checked
through the oracle's layout.
"""
import numpy as np
import pytest
import torch

from moe_overlap_b200 import _lib
from moe_overlap_b200.ep import LocalGroup
from oracle import ep as oep
from tests._inputs import to_storage

pytestmark = pytest.mark.gpu


def routing(world, tokens, num_experts, topk, seed, hidden=256, drop=0.05):
    g = torch.Generator().manual_seed(seed)
    xs, idxs, ws = [], [], []
    for r in range(world):
        xs.append(torch.randn(tokens, hidden, generator=g).to(torch.bfloat16))
        scores = torch.rand(tokens, num_experts, generator=g)
        idx = torch.topk(scores, topk, dim=-1).indices.to(torch.int64)
        idx[torch.rand(tokens, topk, generator=g) < drop] = -1
        idxs.append(idx)
        ws.append(torch.rand(tokens, topk, generator=g).to(torch.float32))
    return xs, idxs, ws


def test_dispatch_layout_matches_oracle(cuda_device):
    lib = _lib.load()
    xs, idxs, _ = routing(1, 3000, 16, 4, seed=1)
    idx = idxs[0].to(cuda_device)
    for world in (1, 2, 4, 8):
        per_rank = torch.empty(world, dtype=torch.int32, device=cuda_device)
        per_expert = torch.empty(16, dtype=torch.int32, device=cuda_device)
        in_rank = torch.empty(3000, world, dtype=torch.bool, device=cuda_device)
        rc = lib.moe_ep_dispatch_layout(idx.data_ptr(), 3000, 4, 16, world, per_rank.data_ptr(),
                                        per_expert.data_ptr(), in_rank.data_ptr(),
                                        torch.cuda.current_stream().cuda_stream)
        assert rc == 0
        want = oep.dispatch_layout(idxs[0].numpy(), 16, world)
        assert np.array_equal(per_rank.cpu().numpy(), want[0])
        assert np.array_equal(per_expert.cpu().numpy(), want[1])
        assert np.array_equal(in_rank.cpu().numpy(), want[2])


@pytest.mark.parametrize("world,tokens,topk,num_experts", [
    (1, 700, 2, 16), (2, 513, 2, 16), (4, 300, 3, 16), (8, 257, 2, 16), (8, 64, 8, 64)])
def test_dispatch_combine_match_oracle(cuda_device, world, tokens, topk, num_experts):
    hidden = 256
    xs, idxs, ws = routing(world, tokens, num_experts, topk, seed=world * 100 + topk, hidden=hidden)
    cap = world * tokens * topk
    grp = LocalGroup(world, num_experts, hidden, tokens, topk, cap, num_blocks=7)
    recv, send_pos = oep.dispatch([to_storage(x) for x in xs], [i.numpy() for i in idxs],
                                  [w.numpy() for w in ws], num_experts)
    try:
        dx = [x.to(cuda_device) for x in xs]
        di = [i.to(cuda_device) for i in idxs]
        dw = [w.to(cuda_device) for w in ws]
        for weighted in (False, True):
            slot, epoch = grp.dispatch(dx, di, dw, pad_rows=True)
            torch.cuda.synchronize()
            assert int(grp.status.item()) == 0, _lib.status_string(int(grp.status.item()))
            ys = []
            for d, ep in enumerate(grp.eps):
                v = ep.slots[slot]
                want = recv[d]
                n = int(want["offsets"][-1])
                assert np.array_equal(v.expert_offsets.cpu().numpy(), want["offsets"])
                assert np.array_equal(to_storage(v.recv_x[:n]), want["x"])
                assert np.array_equal(v.recv_topk_idx[:n, :topk].cpu().numpy(), want["topk_idx"])
                assert np.array_equal(v.recv_topk_weights[:n, :topk].cpu().numpy(),
                                      want["topk_weights"])
                assert np.array_equal(v.recv_src[:n, 0].cpu().numpy(), want["src_rank"])
                assert np.array_equal(v.recv_src[:n, 1].cpu().numpy(), want["src_token"])
                assert bool((v.recv_topk_idx[n:] == -1).all())  # padded rows
                # DeepEP invariants: local ids in {-1} u [0, E/W), per-expert counts.
                ids = v.recv_topk_idx[:n, :topk]
                assert bool(((ids == -1) | ((ids >= 0) & (ids < num_experts // world))).all())
                for le, c in enumerate(np.diff(want["offsets"])):
                    assert int((ids == le).sum()) == c
                # Expert outputs for the combine: a deterministic function of the rows.
                y = (v.recv_x[:n].float() * (1.5 + d) - 0.25).to(torch.bfloat16)
                v.expert_out[:n].copy_(y)
                ys.append(to_storage(y))
            for r, ep in enumerate(grp.eps):
                got = ep.slots[slot].send_pos[: tokens * topk].view(tokens, topk).cpu().numpy()
                assert np.array_equal(got, send_pos[r])
            outs = [torch.empty(tokens, hidden, dtype=torch.bfloat16, device=cuda_device)
                    for _ in range(world)]
            grp.combine(di, dw, slot, epoch, weighted, outs)
            torch.cuda.synchronize()
            assert int(grp.status.item()) == 0
            want = oep.combine(ys, [i.numpy() for i in idxs], send_pos, num_experts,
                               weights=[w.numpy() for w in ws] if weighted else None)
            for r in range(world):
                assert np.array_equal(to_storage(outs[r]), want[r]), (weighted, r)
    finally:
        grp.close()


def test_two_slots_alternate_and_epochs_advance(cuda_device):
    world, tokens, topk, hidden = 4, 200, 2, 128
    grp = LocalGroup(world, 16, hidden, tokens, topk, world * tokens * topk, num_blocks=3)
    try:
        seen = []
        for it in range(5):
            xs, idxs, ws = routing(world, tokens, 16, topk, seed=50 + it, hidden=hidden)
            slot, epoch = grp.dispatch([x.to(cuda_device) for x in xs],
                                       [i.to(cuda_device) for i in idxs],
                                       [w.to(cuda_device) for w in ws])
            torch.cuda.synchronize()
            assert int(grp.status.item()) == 0
            recv, _ = oep.dispatch([to_storage(x) for x in xs], [i.numpy() for i in idxs],
                                   [w.numpy() for w in ws], 16)
            for d, ep in enumerate(grp.eps):
                n = int(recv[d]["offsets"][-1])
                assert np.array_equal(to_storage(ep.slots[slot].recv_x[:n]), recv[d]["x"])
                assert ep.received_rows(slot, epoch) == n
            seen.append((slot, epoch))
        assert [s for s, _ in seen] == [1, 0, 1, 0, 1] and [e for _, e in seen] == [1, 2, 3, 4, 5]
    finally:
        grp.close()


def test_capacity_overflow_is_reported_not_written(cuda_device):
    world, tokens, topk, hidden = 2, 300, 2, 64
    xs, idxs, ws = routing(world, tokens, 8, topk, seed=9, hidden=hidden, drop=0.0)
    grp = LocalGroup(world, 8, hidden, tokens, topk, max_recv_rows=40, num_blocks=4)
    try:
        grp.dispatch([x.to(cuda_device) for x in xs], [i.to(cuda_device) for i in idxs],
                     [w.to(cuda_device) for w in ws])
        torch.cuda.synchronize()
        assert int(grp.status.item()) == _lib.MOE_ERR_CAPACITY
        for ep in grp.eps:
            assert int(ep.slots[1].expert_offsets[-1]) == 0
            with pytest.raises(_lib.MoeError):
                ep.received_rows(1, 1)
    finally:
        grp.close()


def test_wait_that_nobody_satisfies_times_out_with_status(cuda_device):
    """Rank 1 never posts its counts: rank 0's bounded wait must expire and report."""
    world, tokens, topk, hidden = 2, 64, 2, 64
    xs, idxs, ws = routing(world, tokens, 8, topk, seed=3, hidden=hidden)
    grp = LocalGroup(world, 8, hidden, tokens, topk, world * tokens * topk, num_blocks=2)
    try:
        ep0 = grp.eps[0]
        x, i, w = xs[0].to(cuda_device), idxs[0].to(cuda_device), ws[0].to(cuda_device)
        status = torch.zeros(1, dtype=torch.int32, device=cuda_device)
        ep0.dispatch_begin(x, i, w, 1, 1, status)
        ep0.dispatch_scatter(x, i, w, 1, 1, 2, False, 50_000_000, status)  # 50 ms bound
        torch.cuda.synchronize()
        assert int(status.item()) == _lib.MOE_ERR_TIMEOUT
        # The context is still usable afterwards.
        assert float((torch.ones(4, device=cuda_device) * 2).sum()) == 8.0
    finally:
        grp.close()


@pytest.mark.parametrize("world,align", [(1, 64), (2, 64), (4, 16)])
def test_expert_alignment_pads_segments(cuda_device, world, align):
    tokens, topk, hidden, E = 300, 2, 128, 8
    xs, idxs, ws = routing(world, tokens, E, topk, seed=70 + world, hidden=hidden)
    grp = LocalGroup(world, E, hidden, tokens, topk, world * tokens * topk + E * align, num_blocks=5)
    try:
        slot, epoch = grp.dispatch([x.to(cuda_device) for x in xs], [i.to(cuda_device) for i in idxs],
                                   [w.to(cuda_device) for w in ws], expert_alignment=align)
        torch.cuda.synchronize()
        assert int(grp.status.item()) == 0
        recv, send_pos = oep.dispatch([to_storage(x) for x in xs], [i.numpy() for i in idxs],
                                      [w.numpy() for w in ws], E, expert_alignment=align)
        for d, ep in enumerate(grp.eps):
            v, want = ep.slots[slot], recv[d]
            n = int(want["offsets"][-1])
            assert np.array_equal(v.expert_offsets.cpu().numpy(), want["offsets"])
            assert all(int(o) % align == 0 for o in want["offsets"])
            assert np.array_equal(to_storage(v.recv_x[:n]), want["x"])
            assert np.array_equal(v.recv_topk_idx[:n, :topk].cpu().numpy(), want["topk_idx"])
            assert np.array_equal(v.recv_src[:n, 1].cpu().numpy(), want["src_token"])
        for r, ep in enumerate(grp.eps):
            got = ep.slots[slot].send_pos[: tokens * topk].view(tokens, topk).cpu().numpy()
            assert np.array_equal(got, send_pos[r])
    finally:
        grp.close()


@pytest.mark.parametrize("world", [1, 4])
def test_scale_rows_and_topk_weight_grad_match_oracle(cuda_device, world):
    """scale_rows: received rows are bf16(x * w) bit for bit; topk_weight_grad:
    <grad_out[t], y(t, j)> within fp32 summation-order rounding."""
    tokens, topk, hidden, E = 333, 3, 256, 16
    xs, idxs, ws = routing(world, tokens, E, topk, seed=90 + world, hidden=hidden)
    grp = LocalGroup(world, E, hidden, tokens, topk, world * tokens * topk + E * 64, num_blocks=6)
    try:
        di = [i.to(cuda_device) for i in idxs]
        dw = [w.to(cuda_device) for w in ws]
        slot, epoch = grp.dispatch([x.to(cuda_device) for x in xs], di, dw, pad_rows=True,
                                   expert_alignment=64, scale_rows=True)
        torch.cuda.synchronize()
        assert int(grp.status.item()) == 0
        recv, send_pos = oep.dispatch([to_storage(x) for x in xs], [i.numpy() for i in idxs],
                                      [w.numpy() for w in ws], E, expert_alignment=64,
                                      scale_rows=True)
        ys = []
        for d, ep in enumerate(grp.eps):
            v, want = ep.slots[slot], recv[d]
            n = int(want["offsets"][-1])
            assert np.array_equal(to_storage(v.recv_x[:n]), want["x"])
            y = (v.recv_x[:n].float() * 3.0 - 0.5).to(torch.bfloat16)
            v.expert_out[:n].copy_(y)
            ys.append(to_storage(y))
        g = torch.Generator().manual_seed(5)
        gouts = [torch.randn(tokens, hidden, generator=g).to(torch.bfloat16) for _ in range(world)]
        want = oep.topk_weight_grad([to_storage(t) for t in gouts], ys, [i.numpy() for i in idxs],
                                    send_pos, E)
        for r, ep in enumerate(grp.eps):
            out = torch.empty(tokens, topk, dtype=torch.float32, device=cuda_device)
            ep.topk_weight_grad(gouts[r].to(cuda_device), di[r], slot, out, 5)
            torch.cuda.synchronize()
            got = out.cpu().numpy().astype(np.float64)
            np.testing.assert_allclose(got, want[r], rtol=0, atol=2e-4 * np.abs(want[r]).max() + 1e-6)
            assert np.all(got[send_pos[r] < 0] == 0.0)
    finally:
        grp.close()


def test_device_epochs_match_the_oracle(cuda_device):
    """Epoch 0 (drawn on the device, the graph-capturable mode): after two host-epoch
    dispatches, three more with device epochs move the same rows and combine bit-exactly."""
    world, tokens, topk, hidden, E = 4, 211, 2, 128, 8
    grp = LocalGroup(world, E, hidden, tokens, topk, world * tokens * topk, num_blocks=5)
    try:
        for it in range(5):
            if it == 2:
                grp.use_device_epochs()
            xs, idxs, ws = routing(world, tokens, E, topk, seed=300 + it, hidden=hidden)
            di = [i.to(cuda_device) for i in idxs]
            dw = [w.to(cuda_device) for w in ws]
            slot, epoch = grp.dispatch([x.to(cuda_device) for x in xs], di, dw)
            recv, send_pos = oep.dispatch([to_storage(x) for x in xs], [i.numpy() for i in idxs],
                                          [w.numpy() for w in ws], E)
            ys = []
            for d, ep in enumerate(grp.eps):
                n = int(recv[d]["offsets"][-1])
                assert np.array_equal(ep.slots[slot].expert_offsets.cpu().numpy(), recv[d]["offsets"])
                assert np.array_equal(to_storage(ep.slots[slot].recv_x[:n]), recv[d]["x"])
                y = (ep.slots[slot].recv_x[:n].float() * 2.0 + 1.0).to(torch.bfloat16)
                ep.slots[slot].expert_out[:n].copy_(y)
                ys.append(to_storage(y))
            outs = [torch.empty(tokens, hidden, dtype=torch.bfloat16, device=cuda_device)
                    for _ in range(world)]
            grp.combine(di, dw, slot, epoch, True, outs)
            torch.cuda.synchronize()
            assert int(grp.status.item()) == 0, it
            want = oep.combine(ys, [i.numpy() for i in idxs], send_pos, E,
                               weights=[w.numpy() for w in ws])
            for r in range(world):
                assert np.array_equal(to_storage(outs[r]), want[r]), (it, r)
    finally:
        grp.close()


@pytest.mark.parametrize("world,topk", [(1, 2), (2, 2), (4, 3)])
def test_push_gemm_combine_equals_pull_combine(cuda_device, world, topk):
    """The fused down-projection + combine push (moe_ep_push_gemm + moe_ep_combine_pushed)
    gives bit-for-bit the result of the GEMM into expert_out + the pull combine, and both
    match the oracle (the GEMM within bf16 rounding, the reduction bit-exact)."""
    from moe_overlap_b200.gemm import grouped_gemm
    from oracle import grouped_gemm as og

    tokens, hidden, ffn, E = 257, 128, 192, 8
    per = E // world
    xs, idxs, ws = routing(world, tokens, E, topk, seed=500 + world, hidden=hidden)
    g = torch.Generator().manual_seed(41)
    w1 = [(torch.randn(per, ffn, hidden, generator=g) * 0.05).to(torch.bfloat16) for _ in range(world)]
    w2 = [(torch.randn(per, hidden, ffn, generator=g) * 0.05).to(torch.bfloat16) for _ in range(world)]
    cap = world * tokens * topk
    grp = LocalGroup(world, E, hidden, tokens, topk, cap, num_blocks=6)
    try:
        di = [i.to(cuda_device) for i in idxs]
        dw = [w.to(cuda_device) for w in ws]
        slot, epoch = grp.dispatch([x.to(cuda_device) for x in xs], di, dw)
        torch.cuda.synchronize()
        hs, w2t, ys = [], [], []
        for r, ep in enumerate(grp.eps):
            v = ep.slots[slot]
            n = int(v.expert_offsets[-1])
            h = grouped_gemm(v.recv_x, w1[r].to(cuda_device).transpose(1, 2), v.expert_offsets,
                             activation="gelu")
            hs.append(h)
            w2t.append(w2[r].to(cuda_device).transpose(1, 2))
            grouped_gemm(h, w2t[-1], v.expert_offsets, out=v.expert_out)
            ys.append(to_storage(v.expert_out[:n]))
        outs_pull = [torch.empty(tokens, hidden, dtype=torch.bfloat16, device=cuda_device)
                     for _ in range(world)]
        grp.combine(di, dw, slot, epoch, True, outs_pull)
        grp.push_gemm(hs, w2t, slot, epoch)
        outs_push = [torch.empty(tokens, hidden, dtype=torch.bfloat16, device=cuda_device)
                     for _ in range(world)]
        grp.combine_pushed(di, dw, slot, epoch, True, outs_push)
        torch.cuda.synchronize()
        assert int(grp.status.item()) == 0
        recv, send_pos = oep.dispatch([to_storage(x) for x in xs], [i.numpy() for i in idxs],
                                      [w.numpy() for w in ws], E)
        want = oep.combine(ys, [i.numpy() for i in idxs], send_pos, E, weights=[w.numpy() for w in ws])
        for r in range(world):
            assert torch.equal(outs_push[r], outs_pull[r]), r
            assert np.array_equal(to_storage(outs_pull[r]), want[r]), r
            # the expert rows themselves against the oracle GEMM (bf16 rounding)
            n = int(recv[r]["offsets"][-1])
            yo, _ = og.grouped_gemm(to_storage(hs[r][:n]), to_storage(w2t[r].contiguous()),
                                    recv[r]["offsets"], "bf16")
            from oracle.numerics import bf16_bits_to_f32
            diff = np.abs(bf16_bits_to_f32(ys[r]) - bf16_bits_to_f32(yo))
            assert float(diff.max()) <= 2 ** -7 * float(np.abs(bf16_bits_to_f32(yo)).max()) + 1e-2
    finally:
        grp.close()


@pytest.mark.parametrize("world,align,device_epochs", [(1, 64, False), (2, 64, False), (4, 16, True)])
def test_cached_dispatch_matches_oracle(cuda_device, world, align, device_epochs):
    """A cached re-dispatch of new rows on the previous dispatch's layout equals the
    oracle's dispatch of those rows (scaled by the weights) bit for bit: rows,
    metadata, offsets, padding and send positions; its combine is bit-exact too."""
    tokens, topk, hidden, E = 301, 2, 256, 16
    xs, idxs, ws = routing(world, tokens, E, topk, seed=500 + world, hidden=hidden)
    g = torch.Generator().manual_seed(600 + world)
    x2 = [torch.randn(tokens, hidden, generator=g).to(torch.bfloat16) for _ in range(world)]
    grp = LocalGroup(world, E, hidden, tokens, topk, world * tokens * topk + E * align, num_blocks=6)
    try:
        if device_epochs:
            grp.use_device_epochs()
        di = [i.to(cuda_device) for i in idxs]
        dw = [w.to(cuda_device) for w in ws]
        src_slot, _ = grp.dispatch([x.to(cuda_device) for x in xs], di, dw, pad_rows=True,
                                   expert_alignment=align)
        # Garbage in the target slot's receive rows: padding rows must come out zero.
        for ep in grp.eps:
            ep.slots[1 - src_slot].recv_x.fill_(float("nan"))
        slot, epoch = grp.dispatch_cached([x.to(cuda_device) for x in x2], di, dw, src_slot,
                                          pad_rows=True, scale_rows=True)
        torch.cuda.synchronize()
        assert slot != src_slot
        assert int(grp.status.item()) == 0, _lib.status_string(int(grp.status.item()))
        recv, send_pos = oep.dispatch([to_storage(x) for x in x2], [i.numpy() for i in idxs],
                                      [w.numpy() for w in ws], E, expert_alignment=align,
                                      scale_rows=True)
        ys = []
        for d, ep in enumerate(grp.eps):
            v, want = ep.slots[slot], recv[d]
            n = int(want["offsets"][-1])
            assert np.array_equal(v.expert_offsets.cpu().numpy(), want["offsets"])
            assert np.array_equal(to_storage(v.recv_x[:n]), want["x"])
            assert np.array_equal(v.recv_topk_idx[:n, :topk].cpu().numpy(), want["topk_idx"])
            assert np.array_equal(v.recv_topk_weights[:n, :topk].cpu().numpy(), want["topk_weights"])
            assert np.array_equal(v.recv_src[:n, 0].cpu().numpy(), want["src_rank"])
            assert np.array_equal(v.recv_src[:n, 1].cpu().numpy(), want["src_token"])
            assert bool((v.recv_topk_idx[n:] == -1).all())
            y = (v.recv_x[:n].float() * 0.75 + 0.125).to(torch.bfloat16)
            v.expert_out[:n].copy_(y)
            ys.append(to_storage(y))
        for r, ep in enumerate(grp.eps):
            got = ep.slots[slot].send_pos[: tokens * topk].view(tokens, topk).cpu().numpy()
            assert np.array_equal(got, send_pos[r])
        outs = [torch.empty(tokens, hidden, dtype=torch.bfloat16, device=cuda_device)
                for _ in range(world)]
        grp.combine(di, dw, slot, epoch, False, outs)
        torch.cuda.synchronize()
        assert int(grp.status.item()) == 0
        want = oep.combine(ys, [i.numpy() for i in idxs], send_pos, E)
        for r in range(world):
            assert np.array_equal(to_storage(outs[r]), want[r]), r
    finally:
        grp.close()


def test_dispatcher_cached_dispatch_api(cuda_device):
    """DeepEPDispatcher.dispatch(x, handle=...) (world 1): same rows as a full
    dispatch with the handle's routing; misuse is rejected on the host."""
    from moe_overlap_b200.deep_ep_comm import DeepEPDispatcher

    tokens, topk, hidden, E = 257, 2, 128, 8
    xs, idxs, ws = routing(1, tokens, E, topk, seed=77, hidden=hidden)
    x2 = torch.randn(tokens, hidden, generator=torch.Generator().manual_seed(78)).to(torch.bfloat16)
    disp = DeepEPDispatcher(None, hidden, E, num_sms=8, max_tokens_per_rank=tokens, max_top_k=topk)
    try:
        idx, w = idxs[0].to(cuda_device), ws[0].to(cuda_device)
        first = disp.dispatch(xs[0].to(cuda_device), idx, w)
        with pytest.raises(ValueError):
            disp.dispatch(x2.to(cuda_device), idx, w, handle=first.handle)
        with pytest.raises(ValueError):
            disp.dispatch(x2[:-1].to(cuda_device), handle=first.handle)
        again = disp.dispatch(x2.to(cuda_device), handle=first.handle)
        again.event.current_stream_wait()
        torch.cuda.synchronize()
        recv, pos = oep.dispatch([to_storage(x2)], [idxs[0].numpy()], [ws[0].numpy()], E)
        n = int(recv[0]["offsets"][-1])
        assert again.recv_x.shape[0] == n
        assert np.array_equal(to_storage(again.recv_x), recv[0]["x"])
        assert np.array_equal(again.recv_topk_idx.cpu().numpy(), recv[0]["topk_idx"])
        _, ev = disp.combine(first.recv_x.new_zeros(first.recv_x.shape), first.handle)
        ev.current_stream_wait()
        # the cached handle's slot is now the most recent; an older handle is refused
        with pytest.raises(RuntimeError):
            disp.dispatch(x2.to(cuda_device), handle=first.handle)
        out2, ev2 = disp.combine(again.recv_x.clone(), again.handle)
        ev2.current_stream_wait()
        torch.cuda.synchronize()
        # expert outputs = the received rows: each token comes back summed over its slots
        want = oep.combine([recv[0]["x"]], [idxs[0].numpy()], pos, E)
        assert np.array_equal(to_storage(out2), want[0])
    finally:
        disp.close()
