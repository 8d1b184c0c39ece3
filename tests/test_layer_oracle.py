"""Pins the MoE-layer oracle to SimpleMoE outputs made by the reference itself.

tests/golden/moe_layer_golden.npz comes from tests/golden/make_golden_layer.py,
which runs src/train_moe_baseline.py's SimpleMoE on the CPU in fp32: the
single-process routed path and the torch_a2a expert-parallel path on 2 gloo
ranks.  The oracle's fp32 forward must agree to fp32 rounding, and its router
statistics to 1e-5.
"""
from pathlib import Path

import numpy as np
import pytest

from oracle import moe_layer as ol

G = np.load(Path(__file__).parent / "golden" / "moe_layer_golden.npz")


def test_oracle_layer_matches_reference_local_path():
    out = ol.layer_forward_f32(G["x"], G["router_w"], G["w1"], G["w2"], int(G["top_k"]))
    np.testing.assert_allclose(out, G["out_local"], rtol=1e-4, atol=1e-5)


def test_oracle_layer_matches_reference_expert_parallel_path():
    out = ol.layer_forward_f32(G["x"], G["router_w"], G["w1"], G["w2"], int(G["top_k"]))
    half = out.shape[0] // 2
    np.testing.assert_allclose(out[:half], G["out_a2a_rank0"], rtol=1e-4, atol=1e-5)
    np.testing.assert_allclose(out[half:], G["out_a2a_rank1"], rtol=1e-4, atol=1e-5)


def test_oracle_router_stats_match_reference():
    probs, idx, _ = ol.route(G["x"], G["router_w"], int(G["top_k"]))
    ent, std, cv = ol.router_stats(probs, idx, G["router_w"].shape[0])
    np.testing.assert_allclose([ent, std, cv], G["stats"], rtol=1e-5, atol=1e-6)


def test_oracle_layer_backward_matches_reference_autograd():
    dx, dr, dw1, dw2 = ol.layer_backward_f32(G["x"], G["router_w"], G["w1"], G["w2"],
                                             int(G["top_k"]), G["dout"])
    for got, want in ((dx, G["dx"]), (dr, G["d_router_w"]), (dw1, G["d_w1"]), (dw2, G["d_w2"])):
        np.testing.assert_allclose(got, want, rtol=1e-3, atol=1e-5)


def test_oracle_router_topk_backward_matches_torch_autograd():
    """oracle.topk_backward against torch autograd of softmax -> gather -> (renormalise)
    on the CPU, with and without renormalisation and a bias."""
    import torch
    rng = np.random.default_rng(3)
    for renorm in (False, True):
        z = rng.standard_normal((64, 16)).astype(np.float32) * 2
        bias = rng.standard_normal(16).astype(np.float32) * 0.3
        probs, idx, _ = ol.topk_from_logits(z, 3, bias, renorm)
        dw = rng.standard_normal((64, 3))
        zt = torch.tensor(z, dtype=torch.float64, requires_grad=True)
        p = torch.softmax(zt + torch.tensor(bias, dtype=torch.float64), dim=-1)
        sel = p.gather(1, torch.tensor(idx))
        w = sel / sel.sum(dim=-1, keepdim=True) if renorm else sel
        w.backward(torch.tensor(dw))
        got = ol.topk_backward(probs, idx, dw, renorm)
        np.testing.assert_allclose(got, zt.grad.numpy(), rtol=1e-5, atol=1e-7)


def test_layer_chunk_plan_covers_the_batch():
    from moe_overlap_b200.layer import MoELayer

    class _L:
        pass
    for micro in (64, 300, 1000, 4096):
        for taper in (False, True):
            lay = _L()
            lay.micro, lay.taper = micro, taper
            for t in (0, 1, 63, 64, 65, 999, 1000, 8192, 8193):
                plan = MoELayer.chunk_plan(lay, t)
                assert plan[0][0] == 0 and plan[-1][1] == t
                assert all(a[1] == b[0] for a, b in zip(plan[:-1], plan[1:]))
                assert all(0 < e - s <= micro for s, e in plan) or t == 0


def test_package_classes_define_each_method_once():
    """A second definition of a method name in a class body silently replaces the
    first (it once broke the layer forward); no class in the package may do that."""
    import ast
    from pathlib import Path

    pkg = Path(__file__).resolve().parents[1] / "moe_overlap_b200"
    for path in sorted(pkg.glob("*.py")):
        tree = ast.parse(path.read_text())
        for node in ast.walk(tree):
            if isinstance(node, ast.ClassDef):
                names = [f.name for f in node.body
                         if isinstance(f, (ast.FunctionDef, ast.AsyncFunctionDef))
                         and not any(isinstance(d, ast.Attribute) and d.attr in ("setter", "deleter")
                                     for d in f.decorator_list)]
                dup = {n for n in names if names.count(n) > 1}
                assert not dup, (path.name, node.name, dup)


def test_nvtx_range_is_balanced_and_a_no_op_when_off(monkeypatch):
    """The layer's NVTX ranges (reference names, enabled by enable_nvtx) push and pop
    once each, also when the body raises, and touch nothing when disabled."""
    import torch

    from moe_overlap_b200.layer import nvtx_range

    calls = []
    monkeypatch.setattr(torch.cuda, "is_available", lambda: True)
    monkeypatch.setattr(torch.cuda.nvtx, "range_push", lambda n: calls.append(("push", n)))
    monkeypatch.setattr(torch.cuda.nvtx, "range_pop", lambda: calls.append(("pop",)))
    with nvtx_range("deepep_dispatch_chunk_0", True):
        pass
    with pytest.raises(ValueError):
        with nvtx_range("expert_compute_chunk_0", True):
            raise ValueError("x")
    with nvtx_range("deepep_combine_chunk_0", False):
        pass
    assert calls == [("push", "deepep_dispatch_chunk_0"), ("pop",),
                     ("push", "expert_compute_chunk_0"), ("pop",)]


def test_oracle_topk_takes_the_lowest_ids_for_a_nan_row():
    """A NaN logit makes the row's probabilities NaN; the oracle's stable sort then
    keeps id order, so the row takes experts 0..k-1 (the router kernel matches it)."""
    z = np.random.default_rng(0).normal(size=(3, 16)).astype(np.float32)
    z[1, 5] = np.nan
    with np.errstate(invalid="ignore"):
        probs, idx, _ = ol.topk_from_logits(z, 3, renormalize=True)
    assert idx[1].tolist() == [0, 1, 2]
    assert np.isnan(probs[1]).all() and np.isfinite(probs[[0, 2]]).all()


def test_expert_placement_orders():
    """Placement slots -> global experts: the reference's contiguous sharding, the
    strided one, explicit permutations, and the refusals."""
    import pytest

    from moe_overlap_b200.layer import expert_placement_order

    assert expert_placement_order(16, 2) == list(range(16))
    strided = expert_placement_order(16, 4, "strided")
    assert strided[:4] == [0, 4, 8, 12] and strided[4:8] == [1, 5, 9, 13]
    assert sorted(strided) == list(range(16))
    assert expert_placement_order(16, 1, "strided") == list(range(16))
    assert expert_placement_order(4, 2, [3, 2, 1, 0]) == [3, 2, 1, 0]
    with pytest.raises(ValueError):
        expert_placement_order(16, 3)
    with pytest.raises(ValueError):
        expert_placement_order(4, 2, [0, 0, 1, 2])
    with pytest.raises(ValueError):
        expert_placement_order(4, 2, "round-robin")


def test_balanced_placement_evens_out_zipf_loads():
    """Longest-first placement of Zipf(1.0) expert loads: every rank gets E/W experts,
    and the busiest rank's share drops below the contiguous and strided placements'."""
    from moe_overlap_b200.layer import balanced_placement, expert_placement_order

    loads = [1.0 / (e + 1) for e in range(16)]
    total = sum(loads)

    def busiest(order, world):
        per = 16 // world
        return max(sum(loads[e] for e in order[r * per:(r + 1) * per]) for r in range(world)) / total

    for world in (1, 2, 4, 8):
        order = balanced_placement(loads, world)
        assert sorted(order) == list(range(16))
        assert busiest(order, world) <= busiest(expert_placement_order(16, world), world) + 1e-12
        assert busiest(order, world) <= busiest(expert_placement_order(16, world, "strided"), world) + 1e-12
    assert abs(busiest(balanced_placement(loads, 2), 2) - 0.5) < 0.05
    assert balanced_placement(loads, 2) == balanced_placement(loads, 2)  # deterministic
