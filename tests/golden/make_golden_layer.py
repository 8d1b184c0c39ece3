"""Golden vectors for the MoE layer, produced by the reference's own SimpleMoE.

Run where a checkout of the reference is available, with MOE_REFERENCE_SRC
naming its ``src`` directory:

    MOE_REFERENCE_SRC=<checkout>/src python tests/golden/make_golden_layer.py

Records, on the CPU in fp32:
  * the single-process routed path (src/train_moe_baseline.py:342-348,
    expert_kernel="torch", no shared experts): router weight, expert weights,
    input, output and router stats;
  * the gradients torch autograd gives that same path for a seeded output
    gradient (the reference never runs backward, :524-552, but its local path
    is differentiable): d input, d router weight, d w1 / d w2 per expert;
  * the torch_a2a expert-parallel path (:269-313, 323-341) of the same model
    sharded over 2 gloo ranks (each rank's output for its own tokens).
The fixture pins the numpy layer oracle (oracle/moe_layer.py); nothing on the
GPU box reads the reference.
"""
from __future__ import annotations

import os
import socket
import sys
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent
REF_SRC = Path(os.environ["MOE_REFERENCE_SRC"]) if "MOE_REFERENCE_SRC" in os.environ else None
H, F, E, TOPK, T = 32, 64, 8, 2, 128


def _import_ref():
    if REF_SRC is None:
        raise SystemExit("set MOE_REFERENCE_SRC to the reference checkout's src directory")
    sys.path.insert(0, str(REF_SRC))
    sys.dont_write_bytecode = True
    import train_moe_baseline as tmb  # noqa: PLC0415

    return tmb


def _build_local(tmb):
    torch.manual_seed(1234)
    m = tmb.SimpleMoE(H, F, E, 0, TOPK, ep_group=None, comm_backend="local", expert_kernel="torch")
    x = torch.randn(T, H)
    return m, x


def _a2a_worker(rank, world, port, q):
    import torch.distributed as dist

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    tmb = _import_ref()
    full, x = _build_local(tmb)
    m = tmb.SimpleMoE(H, F, E, 0, TOPK, ep_group=dist.group.WORLD, comm_backend="torch_a2a",
                      expert_kernel="torch", micro_batch_size=64)
    sd = full.state_dict()
    per = E // world
    local = {"router.weight": sd["router.weight"]}
    for le in range(per):
        for w in ("w1", "w2"):
            local[f"routed_experts.{le}.{w}.weight"] = sd[f"routed_experts.{rank * per + le}.{w}.weight"]
    m.load_state_dict(local)
    tokens = x.chunk(world)[rank]
    with torch.no_grad():
        out, _ = m(tokens)
    q.put((rank, out.numpy()))
    dist.barrier()
    dist.destroy_process_group()


def main() -> None:
    tmb = _import_ref()
    m, x = _build_local(tmb)
    with torch.no_grad():
        out, stats = m(x)
    sd = m.state_dict()
    xg = x.clone().requires_grad_(True)
    out_g, _ = m(xg)
    dout = torch.randn(out_g.shape, generator=torch.Generator().manual_seed(77))
    out_g.backward(dout)
    data = {
        "dout": dout.numpy(),
        "dx": xg.grad.numpy(),
        "d_router_w": m.router.weight.grad.numpy(),
        "d_w1": np.stack([m.routed_experts[e].w1.weight.grad.numpy() for e in range(E)]),
        "d_w2": np.stack([m.routed_experts[e].w2.weight.grad.numpy() for e in range(E)]),
        "x": x.numpy(),
        "router_w": sd["router.weight"].numpy(),
        "w1": np.stack([sd[f"routed_experts.{e}.w1.weight"].numpy() for e in range(E)]),
        "w2": np.stack([sd[f"routed_experts.{e}.w2.weight"].numpy() for e in range(E)]),
        "out_local": out.numpy(),
        "stats": np.array([stats.entropy, stats.load_std, stats.load_cv]),
        "top_k": np.array(TOPK),
    }
    import torch.multiprocessing as mp

    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_a2a_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    outs = dict(q.get(timeout=300) for _ in range(2))
    for p in procs:
        p.join(timeout=60)
    data["out_a2a_rank0"] = outs[0]
    data["out_a2a_rank1"] = outs[1]
    path = HERE / "moe_layer_golden.npz"
    np.savez_compressed(path, **data)
    print(f"wrote {path} ({path.stat().st_size} bytes); a2a vs local max diff "
          f"{np.abs(np.concatenate([outs[0], outs[1]]) - out.numpy()).max():.3e}")


if __name__ == "__main__":
    main()
