"""GPU parity of the FP8 dispatch payload against the CPU oracle (oracle/fp8.py, oracle/ep.py).

The e4m3 quantisation, the dequantisation and the FP8 dispatch move or compute
bytes, so every check is bit-exact: the quantiser's e4m3 bytes and scales against
the oracle (itself pinned to DeepEP's per_token_cast_to_fp8 by
tests/test_oracle_fp8.py), the rebuilt bf16 rows against per_token_cast_back's
restatement, and every received e4m3 row, scale row, local id, weight, source tag
and expert offset against the oracle's FP8 dispatch (W ranks emulated on one GPU
by LocalGroup, each phase run for all ranks before the next).  The layer with an
FP8 dispatch must equal, bit for bit, the bf16 layer fed the dequantised tokens.
"""
from pathlib import Path

import numpy as np
import pytest
import torch

from moe_overlap_b200 import _lib
from moe_overlap_b200.ep import LocalGroup
from moe_overlap_b200.fp8 import dequantize_fp8, quantize_fp8
from oracle import ep as oep
from oracle import fp8 as ofp8
from tests._inputs import to_storage

pytestmark = pytest.mark.gpu

GOLDEN = Path(__file__).resolve().parent / "golden" / "fp8_golden.npz"


def _u8(t: torch.Tensor) -> np.ndarray:
    return t.detach().cpu().contiguous().view(torch.uint8).numpy()


def test_quantize_and_dequantize_match_the_oracle(cuda_device):
    g = np.load(GOLDEN)
    gen = torch.Generator().manual_seed(8)
    big = (torch.randn(1500, 2048, generator=gen) * 3).to(torch.bfloat16)
    for bits in (g["x"], to_storage(big)):
        x = torch.from_numpy(bits.view(np.int16)).view(torch.bfloat16).to(cuda_device)
        q, sc = quantize_fp8(x)
        want_q, want_sc = ofp8.quantize_per128(bits)
        assert np.array_equal(_u8(q), want_q)
        assert np.array_equal(sc.cpu().numpy().view(np.uint32), want_sc.view(np.uint32))
        back = dequantize_fp8(q, sc)
        assert np.array_equal(to_storage(back), ofp8.dequantize_per128(want_q, want_sc))
    assert np.array_equal(_u8(quantize_fp8(torch.from_numpy(g["x"].view(np.int16))
                                           .view(torch.bfloat16).to(cuda_device))[0]), g["q"])


def test_dequantize_stops_at_the_device_row_count(cuda_device):
    gen = torch.Generator().manual_seed(9)
    x = torch.randn(40, 256, generator=gen).to(torch.bfloat16).to(cuda_device)
    q, sc = quantize_fp8(x)
    out = torch.full((40, 256), 7.0, dtype=torch.bfloat16, device=cuda_device)
    rows = torch.tensor([23], dtype=torch.int32, device=cuda_device)
    dequantize_fp8(q, sc, out=out, rows=rows)
    want = ofp8.dequantize_per128(_u8(q), sc.cpu().numpy())
    assert np.array_equal(to_storage(out[:23]), want[:23])
    assert bool((out[23:] == 7.0).all())


@pytest.mark.parametrize("world,tokens,topk,num_experts", [(1, 300, 2, 16), (2, 513, 2, 16),
                                                           (4, 200, 3, 16)])
def test_fp8_dispatch_matches_oracle(cuda_device, world, tokens, topk, num_experts):
    hidden = 256
    g = torch.Generator().manual_seed(world * 10 + topk)
    xs, idxs, ws = [], [], []
    for _ in range(world):
        xs.append(torch.randn(tokens, hidden, generator=g).to(torch.bfloat16))
        idx = torch.topk(torch.rand(tokens, num_experts, generator=g), topk).indices.to(torch.int64)
        idx[torch.rand(tokens, topk, generator=g) < 0.05] = -1
        idxs.append(idx)
        ws.append(torch.rand(tokens, topk, generator=g))
    grp = LocalGroup(world, num_experts, hidden, tokens, topk, world * tokens * topk, num_blocks=7)
    try:
        qs, scs = zip(*[quantize_fp8(x.to(cuda_device)) for x in xs])
        di = [i.to(cuda_device) for i in idxs]
        dw = [w.to(cuda_device) for w in ws]
        slot, _ = grp.dispatch_fp8(list(qs), list(scs), di, dw)
        torch.cuda.synchronize()
        assert int(grp.status.item()) == 0, _lib.status_string(int(grp.status.item()))
        recv, send_pos = oep.dispatch_fp8([_u8(q) for q in qs], [s.cpu().numpy() for s in scs],
                                          [i.numpy() for i in idxs], [w.numpy() for w in ws],
                                          num_experts)
        for d, ep in enumerate(grp.eps):
            v, want = ep.slots[slot], recv[d]
            n = int(want["offsets"][-1])
            assert np.array_equal(v.expert_offsets.cpu().numpy(), want["offsets"])
            assert np.array_equal(_u8(v.recv_fp8[:n]), want["x_fp8"])
            assert np.array_equal(v.recv_scales[:n].cpu().numpy().view(np.uint32),
                                  want["x_scales"].view(np.uint32))
            assert np.array_equal(v.recv_topk_idx[:n, :topk].cpu().numpy(), want["topk_idx"])
            assert np.array_equal(v.recv_topk_weights[:n, :topk].cpu().numpy(), want["topk_weights"])
            src = v.recv_src[:n].cpu().numpy()
            assert np.array_equal(src[:, 0], want["src_rank"]) and np.array_equal(src[:, 1], want["src_token"])
        for r, ep in enumerate(grp.eps):
            t, k = idxs[r].shape
            assert np.array_equal(ep.slots[slot].send_pos[:t * k].cpu().numpy().reshape(t, k), send_pos[r])
    finally:
        grp.close()


def test_dispatcher_fp8_api_single_rank(cuda_device):
    from moe_overlap_b200.deep_ep_comm import DeepEPDispatcher

    tokens, hidden, experts, topk = 640, 256, 8, 2
    g = torch.Generator().manual_seed(12)
    x = torch.randn(tokens, hidden, generator=g).to(torch.bfloat16).to(cuda_device)
    idx = torch.topk(torch.rand(tokens, experts, generator=g), topk).indices.to(cuda_device)
    w = torch.rand(tokens, topk, generator=g).to(cuda_device)
    disp = DeepEPDispatcher(None, hidden, experts, num_sms=16, max_tokens_per_rank=tokens,
                            max_top_k=topk)
    try:
        with pytest.raises(RuntimeError):  # the reference wrapper's bf16-only dispatch
            disp.dispatch(quantize_fp8(x), idx, w)
        res = disp.dispatch_fp8(quantize_fp8(x), idx, w)
        res.event.current_stream_wait()
        rq, rs = res.recv_x
        assert rq.dtype == torch.float8_e4m3fn and rs.shape == (rq.shape[0], hidden // 128)
        rows = dequantize_fp8(rq, rs)
        src = res.recv_src[:, 1].long()
        want = dequantize_fp8(*quantize_fp8(x))[src]
        assert torch.equal(rows, want)
        out, ev = disp.combine(rows, res.handle)
        ev.current_stream_wait()
        torch.cuda.synchronize()
        assert out.shape == (tokens, hidden)
    finally:
        disp.close()


def test_layer_with_fp8_dispatch_equals_bf16_layer_on_dequantised_tokens(cuda_device):
    from moe_overlap_b200.layer import MoELayer

    tokens, hidden, ffn, experts, topk = 1024, 256, 512, 8, 2
    g = torch.Generator().manual_seed(21)
    x = torch.randn(tokens, hidden, generator=g).to(torch.bfloat16).to(cuda_device)
    ref = MoELayer(hidden, ffn, experts, topk, micro_batch_size=512, num_comm_sms=8).init_random(0.05, 4)
    f8 = MoELayer(hidden, ffn, experts, topk, micro_batch_size=512, num_comm_sms=8,
                  dispatch_fp8=True).init_random(0.05, 4)
    try:
        routing = ref.route(x)
        x_deq = dequantize_fp8(*quantize_fp8(x))
        want, _ = ref(x_deq, routing=routing)
        got, _ = f8(x, routing=routing)
        torch.cuda.synchronize()
        assert torch.equal(got, want)
    finally:
        ref.close()
        f8.close()
