"""GPU parity of the routed MoE layer (router -> dispatch -> GEMMs -> weighted combine).

Two references:
  * the reference's own SimpleMoE output (tests/golden/moe_layer_golden.npz, fp32
    on the CPU), compared with the reference's correctness rule
    max_abs <= 5e-2 and rel_mean <= 5e-2 (src/train_moe_baseline.py:40-41, 719);
  * the oracle at this pipeline's rounding points (oracle/moe_layer.py,
    layer_forward_bf16) for the same routing: at most 1 % of elements may differ
    by more than one bf16 ulp, and none by more than 2^-6 of the magnitude of the
    terms it sums (sum_j |w_j y_j|) + 1e-3, since a one-ulp difference in a large
    expert output survives a near-cancelling weighted sum.
Routing itself is compared with the oracle's router (bf16 logits, fp32 softmax,
as under the reference's autocast): identical expert choices except on near-ties,
where the k-th and (k+1)-th probabilities differ by less than 1 % relative (a
one-ulp flip of a bf16 logit from a different summation order).
"""
from pathlib import Path

import numpy as np
import pytest
import torch

from moe_overlap_b200.layer import MoELayer
from oracle import moe_layer as ol
from oracle.numerics import bf16_bits_to_f32
from tests._inputs import to_storage

pytestmark = pytest.mark.gpu
G = np.load(Path(__file__).parent / "golden" / "moe_layer_golden.npz")


def _bits(t: torch.Tensor) -> np.ndarray:
    return to_storage(t.detach().cpu())


def _close_to_oracle(out: torch.Tensor, want_bits: np.ndarray, magnitude: np.ndarray):
    got = bf16_bits_to_f32(_bits(out)).astype(np.float64)
    want = bf16_bits_to_f32(want_bits).astype(np.float64)
    diff = np.abs(got - want)
    ulp = np.exp2(np.floor(np.log2(np.maximum(np.abs(want), 2.0 ** -30))) - 7)
    assert float(np.mean(diff > ulp * 1.0001)) <= 0.01, float(np.mean(diff > ulp * 1.0001))
    bound = 2.0 ** -6 * np.maximum(np.abs(want), magnitude.astype(np.float64)) + 1e-3
    assert bool(np.all(diff <= bound)), float((diff / bound).max())


def _layer_from_golden(micro):
    E, F_, H = G["w1"].shape
    layer = MoELayer(H, F_, E, int(G["top_k"]), micro_batch_size=micro, num_comm_sms=4)
    sd = {"router.weight": torch.from_numpy(G["router_w"])}
    for e in range(E):
        sd[f"routed_experts.{e}.w1.weight"] = torch.from_numpy(G["w1"][e])
        sd[f"routed_experts.{e}.w2.weight"] = torch.from_numpy(G["w2"][e])
    return layer.load_reference_state_dict(sd)


def test_layer_matches_reference_simplemoe(cuda_device):
    layer = _layer_from_golden(micro=48)
    x = torch.from_numpy(G["x"]).to(cuda_device)
    out, stats = layer(x, return_stats=True)
    torch.cuda.synchronize()
    ref = torch.from_numpy(G["out_local"]).float()
    diff = (out.float().cpu() - ref).abs()
    max_abs, rel_mean = float(diff.max()), float(diff.mean() / ref.abs().mean().clamp_min(1e-8))
    assert max_abs <= 5e-2 and rel_mean <= 5e-2, (max_abs, rel_mean)
    np.testing.assert_allclose([stats.entropy, stats.load_std, stats.load_cv], G["stats"],
                               rtol=2e-2, atol=1e-3)
    layer.close()


def _check_against_oracle(layer, x, renormalize=False, router_b=None):
    probs, idx, w = layer.route(x)
    out, _ = layer(x, routing=(probs, idx, w))
    torch.cuda.synchronize()
    x_bits = _bits(x)
    # Routing: same experts as the oracle's router except on near-ties.
    o_probs, o_idx, _ = ol.route(bf16_bits_to_f32(x_bits), bf16_bits_to_f32(_bits(layer.router_w)),
                                 layer.top_k, router_b, renormalize, bf16_logits=True)
    p_sorted = np.sort(o_probs, axis=-1)[:, ::-1]
    rel_gap = (p_sorted[:, layer.top_k - 1] - p_sorted[:, layer.top_k]) / p_sorted[:, layer.top_k - 1]
    same = (np.sort(idx.cpu().numpy(), axis=-1) == np.sort(o_idx, axis=-1)).all(axis=-1)
    assert float(np.mean(same)) >= 0.99, float(np.mean(same))
    assert bool(np.all(same | (rel_gap < 1e-2))), int((~same & (rel_gap >= 1e-2)).sum())
    want, mag = ol.layer_forward_bf16(x_bits, idx.cpu().numpy(), w.cpu().numpy(), _bits(layer.w1),
                                      _bits(layer.w2), return_magnitude=True)
    _close_to_oracle(out, want, mag)
    return out


def test_layer_matches_oracle_and_is_chunking_invariant(cuda_device):
    g = torch.Generator().manual_seed(5)
    x = torch.randn(1000, 256, generator=g).to(torch.bfloat16).to(cuda_device)
    outs = []
    for micro in (1000, 300, 64):
        layer = MoELayer(256, 512, 16, 2, micro_batch_size=micro, num_comm_sms=8).init_random(seed=3)
        outs.append(_check_against_oracle(layer, x))
        layer.close()
    assert torch.equal(outs[0], outs[1]) and torch.equal(outs[0], outs[2])


def test_layer_renormalised_and_biased_routing(cuda_device):
    g = torch.Generator().manual_seed(6)
    x = torch.randn(512, 128, generator=g).to(torch.bfloat16).to(cuda_device)
    layer = MoELayer(128, 256, 8, 2, renormalize=True, router_bias=True, micro_batch_size=200,
                     num_comm_sms=4).init_random(seed=4)
    bias = (torch.arange(8, dtype=torch.float32) * -0.3)
    layer.router_b.copy_(bias)
    _check_against_oracle(layer, x, renormalize=True, router_b=bias.numpy())
    layer.close()


def test_layer_full_width_config4_chunk(cuda_device):
    """One 4096-token chunk of BASELINE config 4's shapes (H=2048, F=8192, 16 experts, top-2)."""
    g = torch.Generator().manual_seed(7)
    x = torch.randn(4096, 2048, generator=g).to(torch.bfloat16).to(cuda_device)
    layer = MoELayer(2048, 8192, 16, 2, renormalize=True, micro_batch_size=4096,
                     num_comm_sms=16).init_random(seed=8)
    _check_against_oracle(layer, x, renormalize=True)
    layer.close()


def test_forward_graph_replays_the_eager_forward(cuda_device):
    """The chunk-pipelined forward captured as one CUDA graph (device-drawn exchange
    epochs) reproduces the eager forward bit for bit, for the captured and new data."""
    from moe_overlap_b200.layer import ForwardGraph

    g = torch.Generator().manual_seed(17)
    xs = [torch.randn(2048, 256, generator=g).to(torch.bfloat16).to(cuda_device) for _ in range(2)]
    layer = MoELayer(256, 512, 16, 2, micro_batch_size=512, num_comm_sms=16).init_random(seed=5)
    want = [layer(x)[0].clone() for x in xs]
    x_static = xs[0].clone()
    fg = ForwardGraph(layer, x_static)
    for rep, i in enumerate((0, 1, 0)):
        x_static.copy_(xs[i])
        fg.replay()
        torch.cuda.synchronize()
        assert torch.equal(fg.out, want[i]), rep
    # The captured graph's kernels, counted by name: four chunks, each with at least
    # its two GEMMs and its exchange kernels from this library, beside torch's own.
    kc = fg.kernel_counts
    assert kc is not None
    assert 4 * 2 <= kc["ours"] <= kc["total"]
    layer.close()


def test_forward_timeline_marks_every_phase_in_order(cuda_device):
    """forward(timeline=...) records start/end, one dispatch end per chunk, each
    chunk's GEMM span and combine end, and leaves the output bit-identical."""
    g = torch.Generator().manual_seed(23)
    x = torch.randn(2048, 256, generator=g).to(torch.bfloat16).to(cuda_device)
    layer = MoELayer(256, 512, 16, 2, micro_batch_size=512, num_comm_sms=16).init_random(seed=6)
    want = layer(x)[0].clone()
    marks = []
    got = layer(x, timeline=marks)[0]
    torch.cuda.synchronize()
    assert torch.equal(got, want)
    names = [n for n, _ in marks]
    chunks = len(layer.chunk_plan(x.shape[0]))
    assert names[0] == "start" and names[-1] == "end"
    for i in range(chunks):
        assert f"dispatch{i}_end" in names and f"combine{i}_end" in names
        assert names.index(f"gemm{i}_start") < names.index(f"gemm{i}_end")
    ev = dict(marks)
    assert ev["start"].elapsed_time(ev["end"]) >= 0.0
    for i in range(chunks):
        assert ev[f"gemm{i}_start"].elapsed_time(ev[f"gemm{i}_end"]) >= 0.0
    layer.close()


def test_permuted_expert_placement_gives_the_same_output(cuda_device):
    """A layer holding its experts in another order (relabelled before each dispatch,
    weights following) computes every row exactly as before: same bits."""
    from moe_overlap_b200.layer import MoELayer

    tokens, hidden, ffn, experts, topk = 1024, 256, 512, 8, 2
    g = torch.Generator().manual_seed(51)
    x = torch.randn(tokens, hidden, generator=g).to(torch.bfloat16).to(cuda_device)
    base = MoELayer(hidden, ffn, experts, topk, micro_batch_size=512, num_comm_sms=8).init_random(0.05, 8)
    perm = MoELayer(hidden, ffn, experts, topk, micro_batch_size=512, num_comm_sms=8,
                    expert_placement=[5, 2, 7, 0, 1, 6, 3, 4]).init_random(0.05, 8)
    try:
        routing = base.route(x)
        want, _ = base(x, routing=routing)
        got, _ = perm(x, routing=routing)
        torch.cuda.synchronize()
        assert torch.equal(got, want)
    finally:
        base.close()
        perm.close()


def test_one_and_two_gemm_streams_give_the_same_output(cuda_device):
    """The forward's chunks on one compute stream or alternating over two (each with
    its own GEMM1 output and work counter): same bits, over several forwards so that
    chunks reuse both streams' buffers and both dispatch slots."""
    from moe_overlap_b200.layer import MoELayer

    tokens, hidden, ffn, experts, topk = 1300, 256, 512, 8, 2
    g = torch.Generator().manual_seed(61)
    x = torch.randn(tokens, hidden, generator=g).to(torch.bfloat16).to(cuda_device)
    one = MoELayer(hidden, ffn, experts, topk, micro_batch_size=256, num_comm_sms=8,
                   gemm_streams=1).init_random(0.05, 9)
    two = MoELayer(hidden, ffn, experts, topk, micro_batch_size=256, num_comm_sms=8,
                   gemm_streams=2).init_random(0.05, 9)
    try:
        assert len(two.compute_streams) == 2 and two.hs[0].data_ptr() != two.hs[1].data_ptr()
        routing = one.route(x)
        want, _ = one(x, routing=routing)
        for _ in range(3):
            got, _ = two(x, routing=routing)
            torch.cuda.synchronize()
            assert torch.equal(got, want)
    finally:
        one.close()
        two.close()
