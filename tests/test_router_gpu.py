"""GPU parity of the router top-k kernels (moe_router_topk / _backward).

Forward against oracle/moe_layer.py topk_from_logits on the same bf16 or fp32
logits: probabilities within 2e-6 relative, the same experts except where the
k-th and (k+1)-th probabilities are within 1e-6 (a different fp32 summation
order), weights within 2e-6.  Backward against oracle topk_backward (float64)
and torch autograd of softmax / gather / renormalisation on the same routing:
max |diff| <= 1e-5 * max|want| + 1e-7.
"""
import numpy as np
import pytest
import torch

from moe_overlap_b200.router import router_topk
from oracle import moe_layer as ol

pytestmark = pytest.mark.gpu


def _logits(t, e, dtype, seed):
    g = torch.Generator().manual_seed(seed)
    return (torch.randn(t, e, generator=g) * 2.0).to(dtype)


@pytest.mark.parametrize("t,e,k,renorm,bias,dtype", [
    (1000, 16, 2, True, False, torch.bfloat16), (777, 16, 2, False, True, torch.bfloat16),
    (513, 8, 1, False, False, torch.float32), (300, 64, 8, True, True, torch.float32),
    (129, 256, 16, True, False, torch.bfloat16), (0, 16, 2, False, False, torch.bfloat16),
    (5, 40, 3, False, True, torch.float32)])
def test_router_topk_forward_and_backward_match_oracle(cuda_device, t, e, k, renorm, bias, dtype):
    logits = _logits(t, e, dtype, seed=t + e + k)
    b = (torch.arange(e, dtype=torch.float32) * -0.1) if bias else None
    dl = logits.to(cuda_device).requires_grad_(True)
    probs, idx, w = router_topk(dl, k, bias=b.to(cuda_device) if b is not None else None,
                                renormalize=renorm)
    g = torch.Generator().manual_seed(5)
    dw = torch.randn(t, k, generator=g)
    w.backward(dw.to(cuda_device))
    torch.cuda.synchronize()
    zf = logits.float().numpy()
    want_p, want_i, want_w = ol.topk_from_logits(zf, k, b.numpy() if b is not None else None, renorm)
    got_p, got_i, got_w = probs.detach().cpu().numpy(), idx.cpu().numpy(), w.detach().cpu().numpy()
    assert got_p.shape == (t, e) and got_i.shape == (t, k)
    if t == 0:
        return
    np.testing.assert_allclose(got_p, want_p, rtol=2e-6, atol=1e-9)
    srt = np.sort(want_p, axis=-1)[:, ::-1]
    gap = srt[:, k - 1] - (srt[:, k] if k < e else -1.0)
    same = (got_i == want_i).all(axis=-1)
    assert bool(np.all(same | (gap < 1e-6))), int((~same).sum())
    ok = same
    np.testing.assert_allclose(got_w[ok], want_w[ok], rtol=2e-6, atol=1e-9)
    # backward against the oracle on the kernel's own routing
    want_d = ol.topk_backward(got_p, got_i, dw.numpy(), renorm)
    got_d = dl.grad.float().cpu().numpy()
    if dtype == torch.float32:
        tol = 1e-5 * np.abs(want_d).max() + 1e-7
        assert float(np.abs(got_d - want_d).max()) <= tol
    else:  # the gradient is returned in the logits' dtype
        tol = 2 ** -8 * np.abs(want_d) + 1e-5 * np.abs(want_d).max() + 1e-7
        assert bool(np.all(np.abs(got_d - want_d) <= tol))
    # and against torch autograd of the same steps with the same expert choice
    z = logits.float().to(cuda_device).requires_grad_(True)
    zb = z + (b.to(cuda_device) if b is not None else 0.0)
    p = torch.softmax(zb, dim=-1)
    sel = p.gather(1, idx)
    ws = sel / sel.sum(dim=-1, keepdim=True) if renorm else sel
    ws.backward(dw.to(cuda_device))
    ref = z.grad.cpu().numpy()
    assert float(np.abs(ref - want_d).max()) <= 1e-5 * np.abs(want_d).max() + 1e-7


def test_router_topk_rejects_bad_shapes(cuda_device):
    from moe_overlap_b200 import MoeError
    with pytest.raises(MoeError):
        router_topk(torch.zeros(4, 300, device=cuda_device), 2)  # more than 256 experts
    with pytest.raises(MoeError):
        router_topk(torch.zeros(4, 8, device=cuda_device), 9)  # top_k > experts


def test_router_topk_nan_row_takes_the_lowest_ids(cuda_device):
    """A row with a NaN logit (all its probabilities NaN) gets experts 0..k-1 as the
    oracle's stable sort does; other rows are unaffected; every id is in range and
    the backward reads only in-range ids."""
    t, e, k = 40, 16, 3
    logits = _logits(t, e, torch.float32, seed=99)
    logits[7, 3] = float("nan")
    dl = logits.to(cuda_device).requires_grad_(True)
    probs, idx, w = router_topk(dl, k, renormalize=True)
    w.backward(torch.ones(t, k, device=cuda_device))
    torch.cuda.synchronize()
    got_i = idx.cpu().numpy()
    assert got_i.min() >= 0 and got_i.max() < e
    with np.errstate(invalid="ignore"):
        want_p, want_i, _ = ol.topk_from_logits(logits.numpy(), k, None, True)
    assert got_i[7].tolist() == [0, 1, 2] == want_i[7].tolist()
    rows = [r for r in range(t) if r != 7]
    np.testing.assert_allclose(probs.detach().cpu().numpy()[rows], want_p[rows], rtol=2e-6, atol=1e-9)
    assert np.isfinite(dl.grad.cpu().numpy()[rows]).all()
