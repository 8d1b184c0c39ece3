"""Multi-process, multi-GPU check of DeepEPDispatcher over CUDA-IPC peer memory.

Launches tests/_ep_worker.py under torchrun on 2 GPUs (and on every GPU of the
box when it has more, up to 8).  Skipped on a single-GPU machine; the same
kernels are covered there by the in-process multi-rank emulation
(tests/test_ep_gpu.py).  NVLS is switched off: the exchange uses plain peer
loads and stores only.
"""
import os
import socket
import subprocess
import sys
from pathlib import Path

import pytest
import torch

pytestmark = pytest.mark.gpu
REPO = Path(__file__).resolve().parents[1]


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worlds() -> list[int]:
    n = torch.cuda.device_count()
    return sorted({2, min(n, 8)}) if n >= 2 else []


def _run(world: int, worker: str, marker: str) -> None:
    if world not in _worlds():
        pytest.skip(f"needs {world} GPUs (have {torch.cuda.device_count()})")
    env = dict(os.environ, NCCL_NVLS_ENABLE="0", MOE_B200_EP_TIMEOUT_S="20",
               PYTHONDONTWRITEBYTECODE="1")
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
           f"--nproc-per-node={world}", "--master-addr", "127.0.0.1",
           "--master-port", str(_free_port()), str(REPO / "tests" / worker)]
    proc = subprocess.run(cmd, cwd=REPO, env=env, capture_output=True, text=True, timeout=300)
    assert proc.returncode == 0, proc.stdout[-4000:] + proc.stderr[-4000:]
    assert proc.stdout.count(marker) == world


@pytest.mark.parametrize("world", [2, 4, 8])
def test_dispatcher_across_processes(world):
    _run(world, "_ep_worker.py", "exchange matches the oracle")


@pytest.mark.parametrize("world", [2, 4, 8])
def test_moe_layer_across_processes(world):
    _run(world, "_layer_worker.py", "moe layer matches the oracle")


@pytest.mark.parametrize("world", [2, 4, 8])
def test_moe_layer_training_across_processes(world):
    _run(world, "_train_worker.py", "training step matches the reference")
