"""One rank of the multi-GPU exchange check; launched by tests/test_ep_multigpu.py via torchrun.

Every rank draws every rank's inputs from one seed, so each can build the
oracle's answer for its own receive buffer and its own combined output.
Exits non-zero on any mismatch.
"""
import os
import sys
from datetime import timedelta
from pathlib import Path

import numpy as np
import torch
import torch.distributed as dist

sys.path.insert(0, str(Path(__file__).resolve().parents[1]))

from moe_overlap_b200 import _lib  # noqa: E402
from moe_overlap_b200.deep_ep_comm import DeepEPDispatcher  # noqa: E402
from oracle import ep as oep  # noqa: E402
from tests._inputs import to_storage  # noqa: E402


def routing(world, tokens, num_experts, topk, seed, hidden):
    g = torch.Generator().manual_seed(seed)
    xs, idxs, ws = [], [], []
    for _ in range(world):
        xs.append(torch.randn(tokens, hidden, generator=g).to(torch.bfloat16))
        idx = torch.topk(torch.rand(tokens, num_experts, generator=g), topk, dim=-1).indices
        idx[torch.rand(tokens, topk, generator=g) < 0.05] = -1
        idxs.append(idx.to(torch.int64))
        ws.append(torch.rand(tokens, topk, generator=g).to(torch.float32))
    return xs, idxs, ws


def expert_fn(x_bits: np.ndarray, rank: int) -> np.ndarray:
    """A deterministic stand-in for expert compute, identical on CPU and GPU."""
    x = torch.from_numpy(x_bits.view(np.int16)).view(torch.bfloat16)
    return to_storage((x.float() * float(rank + 2)).to(torch.bfloat16))


def main() -> None:
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    local = int(os.environ["LOCAL_RANK"])
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist.init_process_group("nccl", device_id=dev, timeout=timedelta(seconds=90))
    num_experts, hidden, tokens, topk = 16, 512, 777, 2
    xs, idxs, ws = routing(world, tokens, num_experts, topk, seed=2024, hidden=hidden)
    recv, send_pos = oep.dispatch([to_storage(x) for x in xs], [i.numpy() for i in idxs],
                                  [w.numpy() for w in ws], num_experts)
    ys = [expert_fn(recv[d]["x"], d) for d in range(world)]
    disp = DeepEPDispatcher(dist.group.WORLD, hidden, num_experts, num_sms=8,
                            max_tokens_per_rank=1024, max_top_k=topk)
    mine = recv[rank]
    n = int(mine["offsets"][-1])
    x, idx, w = xs[rank].to(dev), idxs[rank].to(dev), ws[rank].to(dev)
    for weighted in (False, True):
        for exact in (True, False):
            res = disp.dispatch(x, idx, w, exact_size=exact)
            res.event.current_stream_wait()
            torch.cuda.synchronize()
            _lib.check_status(dev)
            if exact:
                assert res.recv_x.shape[0] == n, (res.recv_x.shape, n)
            assert np.array_equal(res.expert_offsets.cpu().numpy(), mine["offsets"])
            assert np.array_equal(res.num_recv_tokens_per_expert.cpu().numpy(),
                                  np.diff(mine["offsets"]))
            assert np.array_equal(to_storage(res.recv_x[:n]), mine["x"])
            assert np.array_equal(res.recv_topk_idx[:n].cpu().numpy(), mine["topk_idx"])
            assert np.array_equal(res.recv_topk_weights[:n].cpu().numpy(), mine["topk_weights"])
            assert np.array_equal(res.recv_src[:n].cpu().numpy()[:, 0], mine["src_rank"])
            if not exact:
                assert bool((res.recv_topk_idx[n:] == -1).all())
            y = torch.from_numpy(ys[rank].view(np.int16)).view(torch.bfloat16).to(dev)
            if exact:
                out, ev = disp.combine(y, res.handle, weighted=weighted)
            else:  # zero-copy: write the expert rows straight into the exchange buffer
                disp.expert_out_buffer(res.handle)[:n].copy_(y)
                out, ev = disp.combine(disp.expert_out_buffer(res.handle)[:n], res.handle,
                                       weighted=weighted)
            ev.current_stream_wait()
            torch.cuda.synchronize()
            _lib.check_status(dev)
            want = oep.combine(ys, [i.numpy() for i in idxs], send_pos, num_experts,
                               weights=[v.numpy() for v in ws] if weighted else None)[rank]
            assert np.array_equal(to_storage(out), want), (weighted, exact)
    disp.close()
    dist.barrier()
    dist.destroy_process_group()
    print(f"rank {rank}/{world}: exchange matches the oracle", flush=True)


if __name__ == "__main__":
    main()
