"""GPU parity of the routed-expert backward (forward_autograd / RoutedExperts).

Three references:
  * the reference's own autograd gradients of SimpleMoE (tests/golden/
    moe_layer_golden.npz: dx, d router, dW1, dW2 for a fixed dout, fp32 on the
    CPU), compared with the reference's correctness rule scaled to each tensor:
    mean |diff| <= 5e-2 * mean |want| and max |diff| <= 5e-2 * max |want|
    (src/train_moe_baseline.py:40-41 is the rule for outputs; the gradients go
    through bf16 weights and activations here);
  * the oracle at this pipeline's rounding points for a fixed routing
    (oracle/moe_layer.py experts_backward_bf16): at most 1 % of elements more
    than one bf16 ulp away and none further than 2^-6 of the magnitude of the
    terms summed into it (+ 1e-3 of the tensor's largest value), the top-k
    weight gradient within fp32 summation rounding;
  * a plain PyTorch fp32 autograd of the same layer with the same routing, for
    the router gradient and the full dx: norm-relative error <= 2e-2.
"""
from pathlib import Path

import numpy as np
import pytest
import torch
import torch.nn.functional as F

from moe_overlap_b200.layer import MoELayer, RoutedExperts
from oracle import moe_layer as ol
from oracle.numerics import bf16_bits_to_f32
from tests._inputs import to_storage

pytestmark = pytest.mark.gpu
G = np.load(Path(__file__).parent / "golden" / "moe_layer_golden.npz")


def _bits(t):
    return to_storage(t.detach().cpu())


def _close_bf16(got_t, want_bits, mag):
    got = bf16_bits_to_f32(_bits(got_t)).astype(np.float64)
    want = bf16_bits_to_f32(want_bits).astype(np.float64)
    diff = np.abs(got - want)
    ulp = np.exp2(np.floor(np.log2(np.maximum(np.abs(want), 2.0 ** -30))) - 7)
    frac = float(np.mean(diff > ulp * 1.0001))
    assert frac <= 0.01, frac
    bound = 2.0 ** -6 * np.maximum(np.abs(want), mag.astype(np.float64)) + 1e-3 * np.abs(want).max()
    assert bool(np.all(diff <= bound)), float((diff / bound).max())


def _trainable(layer):
    for t in (layer.router_w, layer.w1, layer.w2):
        t.requires_grad_(True)
    return layer


def test_train_gradients_match_reference_autograd(cuda_device):
    E, F_, H = G["w1"].shape
    layer = MoELayer(H, F_, E, int(G["top_k"]), micro_batch_size=256, num_comm_sms=4, training=True)
    sd = {"router.weight": torch.from_numpy(G["router_w"])}
    for e in range(E):
        sd[f"routed_experts.{e}.w1.weight"] = torch.from_numpy(G["w1"][e])
        sd[f"routed_experts.{e}.w2.weight"] = torch.from_numpy(G["w2"][e])
    _trainable(layer.load_reference_state_dict(sd))
    x = torch.from_numpy(G["x"]).to(cuda_device).requires_grad_(True)
    out, _, _ = layer.forward_autograd(x)
    out.backward(torch.from_numpy(G["dout"]).to(cuda_device).to(out.dtype))
    torch.cuda.synchronize()
    for got, key in ((x.grad, "dx"), (layer.router_w.grad, "d_router_w"),
                     (layer.w1.grad, "d_w1"), (layer.w2.grad, "d_w2")):
        want = torch.from_numpy(G[key]).float()
        diff = (got.float().cpu() - want).abs()
        assert float(diff.mean()) <= 5e-2 * float(want.abs().mean()), (key, float(diff.mean()))
        assert float(diff.max()) <= 5e-2 * float(want.abs().max()), (key, float(diff.max()))
    layer.close()


@pytest.mark.parametrize("tokens,hidden,ffn,experts,topk", [
    (700, 256, 512, 8, 2), (1000, 128, 384, 16, 3)])
def test_expert_gradients_match_oracle(cuda_device, tokens, hidden, ffn, experts, topk):
    g = torch.Generator().manual_seed(tokens + topk)
    layer = MoELayer(hidden, ffn, experts, topk, micro_batch_size=tokens, num_comm_sms=6,
                     training=True).init_random(std=0.05, seed=11)
    _trainable(layer)
    x = torch.randn(tokens, hidden, generator=g).to(torch.bfloat16).to(cuda_device)
    _, idx, w = layer.route(x)
    x.requires_grad_(True)
    w = w.detach().clone().requires_grad_(True)
    out = RoutedExperts.apply(x, w, layer.w1, layer.w2, idx, layer)
    dout = torch.randn(tokens, hidden, generator=g).to(torch.bfloat16).to(cuda_device)
    out.backward(dout)
    torch.cuda.synchronize()
    want = ol.experts_backward_bf16(_bits(x), idx.cpu().numpy(), w.detach().cpu().numpy(),
                                    _bits(layer.w1), _bits(layer.w2), _bits(dout))
    _close_bf16(x.grad, want["dx"], want["mag_dx"])
    _close_bf16(layer.w1.grad, want["dw1"], want["mag_dw1"])
    _close_bf16(layer.w2.grad, want["dw2"], want["mag_dw2"])
    dw = w.grad.cpu().numpy().astype(np.float64)
    np.testing.assert_allclose(dw, want["dw"], rtol=0, atol=2e-3 * np.abs(want["dw"]).max() + 1e-6)
    layer.close()


def _torch_fp32_layer(x, router_w, w1, w2, idx, renormalize):
    """fp32 autograd reference of the routed layer for a fixed routing ``idx``."""
    logits = torch.matmul(x.to(torch.bfloat16), router_w.to(torch.bfloat16).t()).float()
    probs = F.softmax(logits, dim=-1)
    w = probs.gather(1, idx)
    if renormalize:
        w = w / w.sum(dim=-1, keepdim=True)
    xf = x.float()
    out = torch.zeros_like(xf)
    for j in range(idx.shape[1]):
        for e in range(w1.shape[0]):
            rows = (idx[:, j] == e).nonzero().squeeze(1)
            if rows.numel():
                y = F.gelu(xf[rows] @ w1[e].t()) @ w2[e].t()
                out = out.index_add(0, rows, w[rows, j:j + 1] * y)
    return out


def test_full_layer_backward_matches_torch_fp32(cuda_device):
    tokens, hidden, ffn, experts, topk = 2048, 256, 1024, 16, 2
    g = torch.Generator().manual_seed(21)
    layer = _trainable(MoELayer(hidden, ffn, experts, topk, renormalize=True, micro_batch_size=tokens,
                                num_comm_sms=8, training=True).init_random(std=0.05, seed=12))
    x = torch.randn(tokens, hidden, generator=g).to(torch.bfloat16).to(cuda_device).requires_grad_(True)
    dout = torch.randn(tokens, hidden, generator=g).to(torch.bfloat16).to(cuda_device)
    out, _, idx = layer.forward_autograd(x)
    out.backward(dout)
    xr = x.detach().float().requires_grad_(True)
    params = [t.detach().float().requires_grad_(True) for t in (layer.router_w, layer.w1, layer.w2)]
    ref = _torch_fp32_layer(xr, *params, idx.to(torch.int64), renormalize=True)
    ref.backward(dout.float())
    torch.cuda.synchronize()
    rel = lambda a, b: float((a.float() - b).norm() / b.norm().clamp_min(1e-12))
    assert rel(out.detach(), ref.detach()) <= 1e-2
    for got, want in ((x.grad, xr.grad), (layer.router_w.grad, params[0].grad),
                      (layer.w1.grad, params[1].grad), (layer.w2.grad, params[2].grad)):
        assert rel(got, want) <= 2e-2, rel(got, want)
    layer.close()


def test_backward_after_another_dispatch_is_rejected(cuda_device):
    layer = _trainable(MoELayer(128, 256, 8, 2, micro_batch_size=256, num_comm_sms=4,
                                training=True).init_random(seed=1))
    x = torch.randn(256, 128, device=cuda_device).to(torch.bfloat16)
    out1, _, _ = layer.forward_autograd(x)
    out2, _, _ = layer.forward_autograd(x)
    with pytest.raises(RuntimeError, match="dispatch"):
        out1.sum().backward()
    out2.float().sum().backward()
    torch.cuda.synchronize()
    assert layer.w1.grad is not None and torch.isfinite(layer.w1.grad.float()).all()
    layer.close()


@pytest.mark.filterwarnings("error:The AccumulateGrad node's stream does not match")
def test_train_step_graph_replays_the_eager_step(cuda_device):
    """A training step captured as a CUDA graph (device-drawn exchange epochs) gives the
    eager step's results on the same data, replay after replay and for new data."""
    from moe_overlap_b200.layer import TrainStepGraph

    tokens, hidden, ffn, experts, topk = 1024, 256, 512, 8, 2
    layer = _trainable(MoELayer(hidden, ffn, experts, topk, renormalize=True, micro_batch_size=tokens,
                                num_comm_sms=8, training=True).init_random(std=0.05, seed=13))
    g = torch.Generator().manual_seed(31)
    batches = [(torch.randn(tokens, hidden, generator=g).to(torch.bfloat16),
                torch.randn(tokens, hidden, generator=g).to(torch.bfloat16)) for _ in range(2)]

    def eager(xh, dh):
        for p in (layer.router_w, layer.w1, layer.w2):
            p.grad = None
        x = xh.to(cuda_device).requires_grad_(True)
        out, _, idx = layer.forward_autograd(x)
        out.backward(dh.to(cuda_device))
        torch.cuda.synchronize()
        return [t.detach().clone() for t in (out, idx, x.grad, layer.router_w.grad, layer.w1.grad,
                                             layer.w2.grad)]

    want = [eager(xh, dh) for xh, dh in batches]
    xs = batches[0][0].to(cuda_device).requires_grad_(True)
    ds = batches[0][1].to(cuda_device)
    step = TrainStepGraph(layer, xs, ds)
    for rep, (xh, dh) in enumerate([batches[0], batches[1], batches[0]]):
        with torch.no_grad():
            xs.copy_(xh.to(cuda_device))
            ds.copy_(dh.to(cuda_device))
        step.replay()
        torch.cuda.synchronize()
        w = want[0 if rep != 1 else 1]
        got = [step.out, step.topk_idx, xs.grad, layer.router_w.grad, layer.w1.grad, layer.w2.grad]
        assert torch.equal(got[0], w[0]) and torch.equal(got[1], w[1]), rep
        for gt, wt in zip(got[2:], w[2:]):
            assert torch.allclose(gt.float(), wt.float(), rtol=1e-2, atol=1e-3), rep
        assert torch.equal(got[4], w[4]) and torch.equal(got[5], w[5]), rep  # our GEMMs: bitwise
    layer.close()
