"""Host-side logic of the multi-rank exchange on world_size-2 gloo ranks (CPU only).

Covers the buffer exchange (each rank ends up with every rank's buffer,
its own pointer at its own index, peers opened from the gathered handles) and
the failure paths a rank sees on the host: a rank that raises before the
exchange makes the others' collective fail within the process-group timeout
instead of hanging.
"""
import os
import socket
from datetime import timedelta

import pytest
import torch.distributed as dist
import torch.multiprocessing as mp


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _init(rank, world, port, timeout_s=30):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=timedelta(seconds=timeout_s))


def _exchange_worker(rank, world, port, q):
    from moe_overlap_b200.deep_ep_comm import exchange_buffers

    _init(rank, world, port)
    own = 0x1000 * (rank + 1)
    opened = []

    def export():
        return f"handle-of-{rank}".encode()

    def import_(h):
        opened.append(h)
        return 0x1000 * (int(h.decode().split("-")[-1]) + 1) + 0xA

    bases = exchange_buffers(dist.group.WORLD, rank, world, own, export, import_)
    q.put((rank, bases, sorted(opened)))
    dist.barrier()
    dist.destroy_process_group()


def test_exchange_buffers_two_gloo_ranks():
    world, port = 2, _free_port()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_exchange_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    results = {}
    for _ in range(world):
        rank, bases, opened = q.get(timeout=120)
        results[rank] = (bases, opened)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    assert results[0] == ([0x1000, 0x200A], [b"handle-of-1"])
    assert results[1] == ([0x100A, 0x2000], [b"handle-of-0"])


def _dying_worker(rank, world, port, q):
    from moe_overlap_b200.deep_ep_comm import exchange_buffers

    _init(rank, world, port, timeout_s=5)
    if rank == 1:
        q.put((rank, "raised"))
        raise SystemExit(3)  # leaves before the exchange
    try:
        exchange_buffers(dist.group.WORLD, rank, world, 1, lambda: b"h", lambda h: 2)
        q.put((rank, "no error"))
    except Exception as exc:  # the collective must fail, not hang
        q.put((rank, type(exc).__name__))


def test_peer_that_leaves_before_exchange_fails_fast():
    world, port = 2, _free_port()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_dying_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    got = dict(q.get(timeout=120) for _ in range(world))
    for p in procs:
        p.join(timeout=60)
    assert got[1] == "raised"
    assert got[0] != "no error"
    assert procs[1].exitcode == 3
