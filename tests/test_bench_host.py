"""Host-side pieces of bench.py: workload shapes, the config-5 gate bias, exchange row
totals, the clock summary and the cross-rank reduction of the end-to-end legs."""
import sys
from pathlib import Path

import numpy as np
import pytest

sys.path.insert(0, str(Path(__file__).resolve().parents[1]))
import bench  # noqa: E402


def test_workload_counts_follow_the_baseline_configs():
    assert bench.workload_counts("gemm_cfg1") == [128] * 8
    assert bench.workload_counts("gemm_cfg2") == [512] * 16
    c3 = bench.workload_counts("gemm_cfg3")
    assert len(c3) == 16 and sum(c3) == 16384
    assert min(c3) == 0                      # at least one expert gets no rows
    assert max(c3) > 0.25 * 16384            # the largest gets over a quarter
    assert bench.workload_counts("gemm_cfg3") == c3  # seeded


def test_zipf_gate_bias_reproduces_zipf_shares():
    """The fitted per-expert bias makes top-2 routing of N(0,1) tokens follow Zipf(1.0)."""
    rng = np.random.default_rng(0)
    # the config-5 gate: H = 2048, N(0, 0.02) weights (logit spread ~0.9)
    router = (rng.standard_normal((16, 2048)) * 0.02).astype(np.float32)
    bias, iters, err = bench.zipf_gate_bias(router, 16, 2)
    assert bias.shape == (16,) and err < 0.05, (iters, err)
    x = rng.standard_normal((16384, 2048)).astype(np.float32)
    z = x @ router.T + bias
    top = np.argpartition(-z, 1, axis=-1)[:, :2]
    share = np.bincount(top.reshape(-1), minlength=16) / top.size
    p = 1.0 / np.arange(1, 17)
    p /= p.sum()
    assert float(np.max(np.abs(share - p) / p)) < 0.1


def test_layer_workloads_match_the_baseline_shapes():
    w = bench.LAYER_WORKLOADS
    assert (w["layer_train"]["tokens"], w["layer_train"]["hidden"], w["layer_train"]["ffn"],
            w["layer_train"]["experts"], w["layer_train"]["top_k"]) == (8 * 2048, 2048, 8192, 16, 2)
    assert w["layer_train"]["renorm"] and not w["layer_train"]["zipf_bias"]
    assert (w["ep_layer"]["tokens"], w["ep_layer"]["ffn"], w["ep_layer"]["top_k"]) == (8 * 1024, 8192, 2)
    assert w["ep_layer"]["zipf_bias"] and not w["ep_layer"]["renorm"]


def test_exchange_row_totals_ignore_rows_kept_locally():
    import torch

    rows = torch.tensor([[13132.0, 3252.0], [13194.0, 3190.0]])  # rows[src, dst]
    out, inbound = bench.exchange_row_totals(rows)
    assert out == [3252.0, 13194.0]
    assert inbound == [13194.0, 3252.0]
    assert rows[0, 0] == 13132.0  # the caller's matrix is left as it was
    out1, in1 = bench.exchange_row_totals(torch.tensor([[5.0]]))
    assert out1 == [0.0] and in1 == [0.0]


def test_clock_summary_skips_idle_samples_and_names_reasons():
    samples = [(1965, 0x1, 120.0),            # idle: left out
               (1965, 0x0, 900.0),
               (1890, 0x4, 1000.0),           # sw_power_cap
               (1965, 0x4 | 0x20, 950.0)]     # + sw_thermal_slowdown
    c = bench.summarize_clocks(samples, 1965)
    assert c["samples"] == 3 and c["sm_max_mhz"] == 1965
    assert c["sm_mhz"] == 1965 and c["power_w_max"] == 1000.0
    assert c["reasons"] == ["sw_power_cap", "sw_thermal_slowdown"]
    assert bench.summarize_clocks([], 1965)["samples"] == 0
    only_idle = bench.summarize_clocks([(300, 0x1, 80.0)], 1965)
    assert only_idle["samples"] == 1 and only_idle["reasons"] == []


def _e2e_rank(rank, world, port, pipe_ms, q):
    import os

    import torch.distributed as dist

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        q.put((rank, bench.reduce_e2e_legs(10.0 + rank, pipe_ms[rank], world, "cpu")))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("pipe_ms,want", [((6.0, 7.0), (11.0, 7.0)), ((6.0, -1.0), (11.0, -1.0))])
def test_e2e_legs_reduce_over_gloo_ranks(pipe_ms, want):
    """Max over ranks; one rank without the pipelined figure makes every rank report -1."""
    import multiprocessing as mp
    import socket

    with socket.socket() as sk:
        sk.bind(("127.0.0.1", 0))
        port = sk.getsockname()[1]
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_e2e_rank, args=(r, 2, port, pipe_ms, q)) for r in range(2)]
    for p in procs:
        p.start()
    got = dict(q.get(timeout=120) for _ in procs)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    assert got[0] == want and got[1] == want


def test_both_arms_print_the_same_gemm_config():
    """The reference arm and the headline describe the workload with one config object."""
    cfg = bench.gemm_config("gemm_cfg2", 148, 1)
    assert cfg == bench.gemm_config("gemm_cfg2", 148, 1)
    assert cfg["rows"] == 8192 and cfg["counts"] == [512] * 16 and cfg["schedule"] == "striped"
    assert bench.gemm_config("gemm_cfg3", 148, 2)["schedule"] == "atomic"


def test_rows_computed_counts_pair_tiles():
    assert bench.rows_computed([512] * 16) == 8192
    assert bench.rows_computed([1, 0, 257]) == 16 + 256 + 16
    assert bench.rows_computed([129, 384]) == 144 + 256 + 128
    assert bench.rows_computed([224, 225]) == 224 + 256
    assert bench.rows_computed(bench.workload_counts("gemm_cfg3")) == 16544


def test_torch_loop_restatement_matches_the_numpy_oracle():
    """oracle/torch_loop.py (the timed CPU reference) agrees with the oracle's fp32 loop
    to one bf16 rounding (both accumulate in fp32 and round once)."""
    import torch

    from oracle import grouped_gemm as og
    from oracle.numerics import to_f32
    from oracle.torch_loop import grouped_gemm_loop, loop_flops
    from tests._inputs import gemm_inputs, to_storage

    counts = [37, 0, 129, 64]
    a, b, off = gemm_inputs(counts, 256, 192, "bf16", seed=3)
    got = grouped_gemm_loop(a, b, off.tolist())
    want, defined = og.grouped_gemm(to_storage(a), to_storage(b), off.numpy(), "bf16")
    g = to_f32(to_storage(got), "bf16")[defined]
    w = to_f32(want, "bf16")[defined]
    assert np.max(np.abs(g - w)) <= 2.0 ** -7 * np.max(np.abs(w)) + 1e-2
    assert loop_flops(a.shape, b.shape, off.tolist()) == 2 * sum(counts) * 256 * 192
    assert loop_flops(a.shape, b.shape, off.tolist(), [2]) == 2 * 129 * 256 * 192
    del torch


def test_triton_reference_leg_reports_an_absent_install(monkeypatch, tmp_path):
    """Without the reference installed under baseline/_ref the Triton comparison is
    reported unavailable with its reason, never timed."""
    monkeypatch.setattr(bench, "REF_DIR", tmp_path / "absent")
    got = bench.triton_reference(run=None, steps=1, warmup=1)
    assert set(got) == {"unavailable"} and "baseline/_ref" in got["unavailable"]


def test_reference_layer_leg_reports_an_absent_install(monkeypatch, tmp_path):
    monkeypatch.setattr(bench, "REF_DIR", tmp_path / "absent")
    got = bench.reference_layer(layer=None, x=None, device=None)
    assert set(got) == {"unavailable"} and "baseline/_ref" in got["unavailable"]
