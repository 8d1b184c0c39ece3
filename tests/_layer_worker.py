"""One rank of the multi-GPU MoE-layer check; launched by tests/test_ep_multigpu.py via torchrun.

Each rank runs the expert-parallel layer on its own tokens and compares its
output with the oracle evaluated on the full model (every rank can rebuild all
experts' weights from the shared seed), for the routing the layer chose.
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
from moe_overlap_b200.layer import MoELayer, random_weights  # noqa: E402
from oracle import moe_layer as ol  # noqa: E402
from oracle.numerics import bf16_bits_to_f32  # noqa: E402
from tests._inputs import to_storage  # noqa: E402


def main() -> None:
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    local = int(os.environ["LOCAL_RANK"])
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist.init_process_group("nccl", device_id=dev, timeout=timedelta(seconds=90))
    H, Fd, E, K, T = 256, 512, 16, 2, 900
    layer = MoELayer(H, Fd, E, K, group=dist.group.WORLD, micro_batch_size=256,
                     num_comm_sms=8).init_random(seed=11)
    g = torch.Generator().manual_seed(100 + rank)
    x = torch.randn(T, H, generator=g).to(torch.bfloat16)
    probs, idx, w = layer.route(x.to(dev))
    out, stats = layer(x.to(dev), return_stats=True, routing=(probs, idx, w))
    torch.cuda.synchronize()
    _lib.check_status(dev)
    _, w1, w2 = random_weights(E, H, Fd, 0.02, 11)
    want, mag = ol.layer_forward_bf16(to_storage(x), idx.cpu().numpy(), w.cpu().numpy(),
                                      to_storage(w1.to(torch.bfloat16)),
                                      to_storage(w2.to(torch.bfloat16)), return_magnitude=True)
    got = bf16_bits_to_f32(to_storage(out.cpu())).astype(np.float64)
    ref = bf16_bits_to_f32(want).astype(np.float64)
    diff = np.abs(got - ref)
    bound = 2.0 ** -6 * np.maximum(np.abs(ref), mag) + 1e-3
    assert bool(np.all(diff <= bound)), float((diff / bound).max())
    ulp = np.exp2(np.floor(np.log2(np.maximum(np.abs(ref), 2.0 ** -30))) - 7)
    assert float(np.mean(diff > ulp * 1.0001)) <= 0.01
    assert stats.load_cv >= 0.0
    # The same layer with tile-granular overlap (expert-ordered dispatch, GEMM tiles
    # waiting per expert for rows that arrive over NVLink) gives the same bits.
    over = MoELayer(H, Fd, E, K, group=dist.group.WORLD, micro_batch_size=256, num_comm_sms=8,
                    overlap_tiles=True).init_random(seed=11)
    for _ in range(2):
        out2, _ = over(x.to(dev), routing=(probs, idx, w))
        torch.cuda.synchronize()
        _lib.check_status(dev)
        assert torch.equal(out2, out), "tile-overlap layer differs from the layer"
    over.close()
    # Strided expert placement (rank r holds experts r, r + W, ...): the same layer
    # with its experts dealt out differently, against the same oracle bound.
    strided = MoELayer(H, Fd, E, K, group=dist.group.WORLD, micro_batch_size=256, num_comm_sms=8,
                       expert_placement="strided").init_random(seed=11)
    out3, _ = strided(x.to(dev), routing=(probs, idx, w))
    torch.cuda.synchronize()
    _lib.check_status(dev)
    got3 = bf16_bits_to_f32(to_storage(out3.cpu())).astype(np.float64)
    diff3 = np.abs(got3 - ref)
    assert bool(np.all(diff3 <= bound)), float((diff3 / bound).max())
    strided.close()
    layer.close()
    dist.barrier()
    dist.destroy_process_group()
    print(f"rank {rank}/{world}: moe layer matches the oracle", flush=True)


if __name__ == "__main__":
    main()
