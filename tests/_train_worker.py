"""One rank of the multi-GPU MoE-layer training check; launched by tests/test_ep_multigpu.py.

Each rank runs forward_autograd + backward of the expert-parallel layer on its
own tokens.  Every rank rebuilds the full model (shared seed) and the batch of
every rank, takes the routing the layers chose (all-gathered), and evaluates a
plain fp32 torch autograd of the whole layer on all tokens.  Its own slice must
match: the output and dx of its tokens, dW1/dW2 of its experts (summed over all
ranks' tokens), and the router gradient from its own tokens; norm-relative error
<= 2e-2 (bf16 weights, activations and exchanged rows).
"""
import os
import sys
from datetime import timedelta
from pathlib import Path

import torch
import torch.distributed as dist
import torch.nn.functional as F

sys.path.insert(0, str(Path(__file__).resolve().parents[1]))

from moe_overlap_b200 import _lib  # noqa: E402
from moe_overlap_b200.layer import MoELayer, random_weights  # noqa: E402


def _reference(x, router_w, w1, w2, idx):
    """fp32 autograd of the routed layer (renormalised top-k) for a fixed routing."""
    logits = torch.matmul(x.to(torch.bfloat16), router_w.to(torch.bfloat16).t()).float()
    p = torch.softmax(logits, dim=-1).gather(1, idx)
    w = p / p.sum(dim=-1, keepdim=True)
    out = torch.zeros_like(x)
    for j in range(idx.shape[1]):
        for e in range(w1.shape[0]):
            rows = (idx[:, j] == e).nonzero().squeeze(1)
            if rows.numel():
                y = F.gelu(x[rows] @ w1[e].t()) @ w2[e].t()
                out = out.index_add(0, rows, w[rows, j:j + 1] * y)
    return out


def main() -> None:
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    local = int(os.environ["LOCAL_RANK"])
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist.init_process_group("nccl", device_id=dev, timeout=timedelta(seconds=90))
    H, Fd, E, K, T = 128, 256, 8, 2, 384
    layer = MoELayer(H, Fd, E, K, group=dist.group.WORLD, renormalize=True, micro_batch_size=T,
                     num_comm_sms=8, training=True).init_random(std=0.05, seed=21)
    for p in (layer.router_w, layer.w1, layer.w2):
        p.requires_grad_(True)
    g = torch.Generator().manual_seed(7)
    xs = [torch.randn(T, H, generator=g).to(torch.bfloat16) for _ in range(world)]
    douts = [torch.randn(T, H, generator=g).to(torch.bfloat16) for _ in range(world)]
    x = xs[rank].to(dev).requires_grad_(True)
    out, _, idx = layer.forward_autograd(x)
    out.backward(douts[rank].to(dev))
    torch.cuda.synchronize()
    _lib.check_status(dev)

    idx_all = [torch.empty_like(idx) for _ in range(world)]
    dist.all_gather(idx_all, idx.contiguous())
    # full model, as every rank's layer drew it (bf16 weights)
    rw, w1, w2 = (t.to(torch.bfloat16).float().to(dev) for t in random_weights(E, H, Fd, 0.05, 21))
    x_all = torch.cat([t.to(dev).float() for t in xs]).requires_grad_(True)
    rw_r, w1_r, w2_r = (t.clone().requires_grad_(True) for t in (rw, w1, w2))
    ref = _reference(x_all, rw_r, w1_r, w2_r, torch.cat(idx_all))
    d_all = torch.cat([t.to(dev).float() for t in douts])
    ref.backward(d_all, retain_graph=True)
    # router gradient from this rank's tokens only
    rw_only = rw.clone().requires_grad_(True)
    mask = torch.zeros(world * T, 1, device=dev)
    mask[rank * T:(rank + 1) * T] = 1.0
    ref2 = _reference(x_all.detach(), rw_only, w1, w2, torch.cat(idx_all))
    ref2.backward(d_all * mask)

    def rel(a, b):
        return float((a.float() - b).norm() / b.norm().clamp_min(1e-12))

    lo, hi = rank * T, (rank + 1) * T
    per = E // world
    checks = {
        "out": rel(out.detach(), ref.detach()[lo:hi]),
        "dx": rel(x.grad, x_all.grad[lo:hi]),
        "dw1": rel(layer.w1.grad, w1_r.grad[rank * per:(rank + 1) * per]),
        "dw2": rel(layer.w2.grad, w2_r.grad[rank * per:(rank + 1) * per]),
        "d_router": rel(layer.router_w.grad, rw_only.grad),
    }
    bad = {k: v for k, v in checks.items() if not v <= 2e-2}
    assert not bad, (rank, bad)
    layer.close()
    dist.barrier()
    dist.destroy_process_group()
    print(f"rank {rank}/{world}: training step matches the reference", flush=True)


if __name__ == "__main__":
    main()
