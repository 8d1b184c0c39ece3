#!/usr/bin/env python
"""Benchmark of the moe_overlap_b200 hot path (driver contract: one JSON line).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--workload gemm_cfg2|gemm_cfg3|gemm_cfg1|ep_layer|layer_fwd|layer_train]

Default workload: BASELINE config 2 -- grouped GEMM forward, 16 experts x 512
rows, H=2048, F=4096, bf16, striped persistent schedule over every SM.  One
"step" is one grouped-GEMM launch over the whole batch; ``value`` is the
TFLOP/s of all ranks together (2*M*K*N algorithmic flops, real rows only)
divided by the device time of the K timed launches (CUDA events on the
launching stream, max over ranks).  L2 is flushed (a 256 MiB write) between
timed launches, outside the events.  ``e2e`` times the same step through the
public ``persistent_grouped_gemm`` call with the activations and offsets
copied from pinned host memory and the result copied back inside the timed
region (expert weights stay resident, as model parameters do), with copy-in,
GEMM and copy-out of consecutive steps overlapped on three streams; the same
steps run back to back on one stream are reported beside it.

The default line carries two more measurements of the same run:
  ``gemm_cfg3``  BASELINE config 3 (16 experts, Zipf(1.2)-skewed 16384 rows, one
                 expert empty, atomic tile queue), timed like the headline;
  ``ep_layer``   BASELINE config 5, the expert-parallel MoE layer (router,
                 dispatch, grouped GEMMs, weighted combine) with the 16 experts
                 sharded over the N ranks of the run: tokens/s of all ranks,
                 rows received per rank, the communication-hidden ratio, and the
                 device time and NVLink rate of every exchange launch.
With N > 1 (torchrun) every rank runs its own copy of the config 2 and 3 GEMMs
(the grouped GEMM has no cross-rank exchange, so scaling is weak and there is
no collective on their data path), and all ranks run config 5 together.

``--impl reference`` times the reference's CPU implementation of the path on
this host's cores: the per-expert torch loop of ``reference_grouped_gemm``
(restated in ``oracle/torch_loop.py``; the reference's Python cannot travel to
the GPU box), over the same workload and configuration as the headline.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import sys
import threading
import time
from pathlib import Path

REPO = Path(__file__).resolve().parent
sys.path.insert(0, str(REPO))

METRIC = "grouped-GEMM TFLOP/s vs bf16 peak"
UNIT = "TFLOP/s"
FALLBACK_PEAK_TFLOPS = 1590.0
PEER_COPY_GBPS = 770.0  # measured peer copy per direction per B200 on this pool

WORKLOADS = {
    # name: (counts builder, k, n, dtype, atomic, description)
    "gemm_cfg2": dict(k=2048, n=4096, dtype="bf16", atomic=False, experts=16,
                      desc="BASELINE config 2: E=16, 512 rows/expert (8192 rows), H=2048, F=4096, bf16, striped"),
    "gemm_cfg3": dict(k=2048, n=4096, dtype="bf16", atomic=True, experts=16,
                      desc="BASELINE config 3: E=16, 16384 Zipf(1.2) rows (one expert empty), H=2048, F=4096, bf16, atomic queue"),
    "gemm_cfg1": dict(k=512, n=1024, dtype="f16", atomic=False, experts=8,
                      desc="BASELINE config 1: E=8, 128 rows/expert, H=512, F=1024, fp16, striped"),
}


LAYER_WORKLOADS = {
    "ep_layer": dict(tokens=8 * 1024, hidden=2048, ffn=8192, experts=16, top_k=2, renorm=False,
                     zipf_bias=True,
                     desc="BASELINE config 5: expert-parallel MoE layer forward, per rank 8x1024 "
                          "tokens, H=2048, F=8192, 16 experts sharded over the ranks, top-2 "
                          "softmax, Zipf(1.0) gate bias"),
    "layer_fwd": dict(tokens=8 * 2048, hidden=2048, ffn=8192, experts=16, top_k=2, renorm=True,
                      zipf_bias=False,
                      desc="BASELINE config 4 forward: MoE layer on one GPU, batch 8 x seq 2048, "
                           "H=2048, FFN 4H, 16 experts, renormalised top-2"),
    "layer_train": dict(tokens=8 * 2048, hidden=2048, ffn=8192, experts=16, top_k=2, renorm=True,
                        zipf_bias=False,
                        desc="BASELINE config 4: MoE layer forward + backward on one GPU, batch 8 x "
                             "seq 2048, H=2048, FFN 4H, 16 experts, renormalised top-2"),
}


def workload_counts(name: str) -> list[int]:
    from tests._inputs import zipf_counts

    if name == "gemm_cfg2":
        return [512] * 16
    if name == "gemm_cfg3":
        return zipf_counts(16384, 16, 1.2, seed=0)
    if name == "gemm_cfg1":
        return [128] * 8
    raise ValueError(name)


def parse_args() -> argparse.Namespace:
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--workload", choices=sorted(WORKLOADS) + sorted(LAYER_WORKLOADS),
                    default="gemm_cfg2")
    ap.add_argument("--comm-sms", type=int, default=148,
                    help="layer workloads: blocks of the dispatch/combine kernels (one per SM "
                         "by default; they run beside the persistent GEMM CTAs)")
    ap.add_argument("--placement", choices=["contiguous", "strided", "balanced"],
                    default="contiguous",
                    help="layer workloads: which experts each rank holds (contiguous: the "
                         "reference's sharding; strided: rank r holds r, r+N, ...; balanced: "
                         "longest-first by the gate's target expert shares)")
    ap.add_argument("--solo-blocks", type=int, default=0,
                    help="layer workloads: blocks of the exchange phases that run alone (default "
                         "four per SM)")
    ap.add_argument("--gemm-streams", type=int, choices=[1, 2], default=2,
                    help="layer workloads: compute streams the forward's chunks alternate over")
    ap.add_argument("--micro-batch", type=int, default=4096,
                    help="layer workloads: tokens per pipelined chunk")
    ap.add_argument("--no-graph", action="store_true",
                    help="layer workloads: time eager steps instead of a captured CUDA graph")
    ap.add_argument("--combine", choices=["auto", "push", "pull"], default="auto",
                    help="layer workloads: GEMM-fused combine push, or GEMM into expert_out + pull "
                         "combine (auto: the layer's default, pull)")
    ap.add_argument("--timeline", action="store_true",
                    help="layer workloads: add per-rank phase-boundary times of one forward")
    ap.add_argument("--nvtx", action="store_true",
                    help="layer workloads: NVTX ranges per chunk, named as the reference's "
                         "(deepep_dispatch_chunk_i, expert_compute_chunk_i, deepep_combine_chunk_i)")
    ap.add_argument("--overlap-tiles", choices=["auto", "on", "off"], default="auto",
                    help="layer workloads: expert-ordered dispatch with GEMM tiles that start per "
                         "expert as its rows land (auto: the layer's default)")
    ap.add_argument("--dispatch-fp8", action="store_true",
                    help="layer forward workloads: dispatch tokens as e4m3 + per-128 scales")
    ap.add_argument("--taper", action="store_true",
                    help="layer workloads: quarter-size first/last chunks instead of equal chunks")
    ap.add_argument("--no-cpu-baseline", action="store_true", help="skip the CPU baseline leg")
    ap.add_argument("--no-e2e", action="store_true", help="skip the end-to-end leg")
    ap.add_argument("--no-extras", action="store_true",
                    help="default workload: skip the gemm_cfg3 and ep_layer measurements")
    return ap.parse_args()


def cpu_cores() -> int:
    try:
        return len(os.sched_getaffinity(0))
    except AttributeError:  # pragma: no cover
        return os.cpu_count() or 1


def load_peaks() -> tuple[float, str]:
    path = REPO / "MEASURED_PEAKS.json"
    try:
        peaks = json.loads(path.read_text())
        return float(peaks["bf16_tflops"]), "measured (MEASURED_PEAKS.json bf16_tflops, burst)"
    except Exception:
        return FALLBACK_PEAK_TFLOPS, "fallback (no MEASURED_PEAKS.json)"


def profiled_traffic(workload: str) -> float | None:
    """DRAM bytes per launch from the committed ncu summary of this workload."""
    path = REPO / "profiles" / f"grouped_gemm_{workload.split('_')[-1]}.ncu.txt"
    try:
        for line in path.read_text().splitlines():
            if line.startswith("dram_bytes_per_launch:"):
                return float(line.split(":", 1)[1].strip())
    except OSError:
        return None
    return None


def gemm_config(name: str, num_sms: int, world: int) -> dict:
    """The ``config`` object of a grouped-GEMM line; both arms print the same one."""
    wl = WORKLOADS[name]
    counts = workload_counts(name)
    rows = int(sum(counts))
    in_mib = (rows * wl["k"] + len(counts) * wl["k"] * wl["n"]) * 2 >> 20
    return {
        "workload": name,
        "description": wl["desc"],
        "rows": rows,
        "counts": counts,
        "num_sms": num_sms,
        "schedule": "atomic" if wl["atomic"] else "striped",
        "l2": "flushed between timed launches (256 MiB write, outside the events); "
              f"inputs also exceed L2 (A+B = {in_mib} MiB)",
        "parallelism": f"replica x{world} (no data-path collective)",
    }


def device_sm_count(local_rank: int = 0) -> int:
    """SMs of this rank's GPU (148 on a B200 when no GPU is visible)."""
    try:
        import torch

        if torch.cuda.is_available():
            return torch.cuda.get_device_properties(local_rank).multi_processor_count
    except Exception:
        pass
    return 148


def rows_computed(counts) -> int:
    """Rows the CTA-pair GEMM multiplies for these expert counts (tensor work incl. padding).

    Every expert's rows are cut into 256-row pair tiles; a last tile of at most
    224 rows runs swapped (the weights take the MMA's 256-row side and the tile's
    rows its N side, rounded up to 16), so it costs its rows rounded up to 16; a
    longer last tile costs 256.
    """
    total = 0
    for c in counts:
        full, tail = divmod(int(c), 256)
        total += 256 * full + (0 if tail == 0 else ((tail + 15) // 16 * 16 if tail <= 224 else 256))
    return total


# ---------------------------------------------------------------- CPU side --
def set_cpu_threads(n: int) -> int:
    import torch

    torch.set_num_threads(n)
    try:
        from threadpoolctl import threadpool_limits

        threadpool_limits(n)
    except Exception:
        pass
    return n


class CpuReference:
    """The reference's CPU grouped GEMM on this host: the per-expert torch loop of
    ``reference_grouped_gemm`` (src/triton_grouped_gemm.py:446-457), restated in
    oracle/torch_loop.py, in the workload's dtype on all host cores."""

    def __init__(self, name: str):
        from oracle.torch_loop import grouped_gemm_loop, loop_flops
        from tests._inputs import gemm_inputs

        wl = WORKLOADS[name]
        self.name, self.dtype = name, wl["dtype"]
        self.counts = workload_counts(name)
        self.a, self.b, off = gemm_inputs(self.counts, wl["k"], wl["n"], wl["dtype"], seed=0)
        self.off = off.tolist()
        self.out = None
        self.experts = [e for e, c in enumerate(self.counts) if c > 0]
        self._loop, self._flops = grouped_gemm_loop, loop_flops

    def step(self, experts=None) -> int:
        """One pass of the loop (all experts, or the given sample); returns its flops."""
        self.out = self._loop(self.a, self.b, self.off, experts, self.out)
        return self._flops(self.a.shape, self.b.shape, self.off, experts)

    def plan(self, n_steps: int, budget_s: float) -> tuple[list | None, str]:
        """The experts one step runs so that ``n_steps`` steps fit in ``budget_s``:
        the whole workload when it fits, else the largest prefix of the experts."""
        self.step(self.experts[:1])  # warm the threads
        t0 = time.perf_counter()
        full_flops = self.step()
        per_flop = (time.perf_counter() - t0) / max(1, full_flops)
        if per_flop * full_flops * n_steps <= budget_s:
            return None, f"the whole workload per step ({len(self.experts)} experts, " \
                         f"{full_flops / 1e9:.1f} GFLOP)"
        sample, flops = [], 0
        for e in self.experts:
            f = self._flops(self.a.shape, self.b.shape, self.off, [e])
            if sample and per_flop * (flops + f) * n_steps > budget_s:
                break
            sample.append(e)
            flops += f
        return sample, f"experts {sample} of {len(self.experts)} per step ({flops / 1e9:.1f} " \
                       f"GFLOP), to keep {n_steps} steps within {budget_s:.0f} s"


def cpu_sample_text(name: str, what: str) -> str:
    return (f"{what} of {name}: per-expert torch matmul loop in {WORKLOADS[name]['dtype']} "
            "(reference_grouped_gemm, src/triton_grouped_gemm.py:446-457, restated in "
            "oracle/torch_loop.py), inputs resident in host memory")


def cpu_baseline(name: str, budget_s: float = 20.0) -> dict:
    """The reference's CPU grouped GEMM timed on this host (bounded sample)."""
    cores = set_cpu_threads(cpu_cores())
    ref = CpuReference(name)
    ref.step(ref.experts[:1])
    done_flops, passes = 0, 0
    t0 = time.perf_counter()
    while True:
        done_flops += ref.step()
        passes += 1
        if time.perf_counter() - t0 > min(budget_s, 3.0) or passes >= 100:
            break
    dt = time.perf_counter() - t0
    return {
        "value": round(done_flops / dt / 1e12, 4),
        "unit": UNIT,
        "cores": cores,
        "kind": "port",
        "sample": cpu_sample_text(name, f"{passes} whole passes ({done_flops / 1e9:.1f} GFLOP in "
                                        f"{dt:.2f} s)"),
    }


def run_reference(args, rank: int) -> None:
    """The reference arm: the reference's CPU implementation of the path, rank 0 only,
    on the headline's workload, metric and configuration."""
    if rank != 0:
        return
    cores = set_cpu_threads(cpu_cores())
    ref = CpuReference(args.workload)
    sample, sample_text = ref.plan(args.steps + args.warmup, budget_s=150.0)
    for _ in range(args.warmup):
        ref.step(sample)
    flops, t0 = 0, time.perf_counter()
    for _ in range(args.steps):
        flops += ref.step(sample)
    dt = time.perf_counter() - t0
    value = flops / dt / 1e12
    sample = cpu_sample_text(args.workload, sample_text)
    line = {
        "impl": "reference",
        "metric": METRIC,
        "value": round(value, 4),
        "unit": UNIT,
        "n_gpus": args.gpus,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": round(dt / max(1, args.steps) * 1e3, 4),
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": WORKLOADS[args.workload]["dtype"],
        "data": "synthetic (seeded N(0,1) activations, N(0,0.02) weights; generated on CPU)",
        "config": gemm_config(args.workload, device_sm_count(), args.gpus),
        "cpu_baseline": {"value": round(value, 4), "unit": UNIT, "cores": cores, "kind": "port",
                         "sample": sample},
        "e2e": {"value": round(value, 4), "unit": UNIT, "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


# ---------------------------------------------------------------- clocks --
_REASONS = {
    0x1: "gpu_idle", 0x2: "applications_clocks_setting", 0x4: "sw_power_cap",
    0x8: "hw_slowdown", 0x10: "sync_boost", 0x20: "sw_thermal_slowdown",
    0x40: "hw_thermal_slowdown", 0x80: "hw_power_brake_slowdown", 0x100: "display_clock_setting",
}


class ClockSampler(threading.Thread):
    """Samples SM clock, power and clock-event reasons through NVML."""

    def __init__(self, torch_device, interval_s: float = 0.002):
        super().__init__(daemon=True)
        self.interval = interval_s
        self.samples: list[tuple[int, int, float]] = []
        self.max_mhz = None
        self._stop_evt = threading.Event()
        self.handle = None
        try:
            import pynvml
            import torch

            pynvml.nvmlInit()
            props = torch.cuda.get_device_properties(torch_device)
            try:
                self.handle = pynvml.nvmlDeviceGetHandleByUUID(f"GPU-{props.uuid}")
            except Exception:
                self.handle = pynvml.nvmlDeviceGetHandleByIndex(torch_device.index or 0)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self.handle, pynvml.NVML_CLOCK_SM)
            self.nvml = pynvml
        except Exception:
            self.handle = None

    def run(self) -> None:
        if self.handle is None:
            return
        nv = self.nvml
        while not self._stop_evt.is_set():
            try:
                sm = nv.nvmlDeviceGetClockInfo(self.handle, nv.NVML_CLOCK_SM)
                try:
                    reasons = nv.nvmlDeviceGetCurrentClocksEventReasons(self.handle)
                except Exception:
                    reasons = nv.nvmlDeviceGetCurrentClocksThrottleReasons(self.handle)
                power = nv.nvmlDeviceGetPowerUsage(self.handle) / 1000.0
                self.samples.append((sm, reasons, power))
            except Exception:
                pass
            time.sleep(self.interval)

    def stop(self) -> dict:
        self._stop_evt.set()
        if self.is_alive():
            self.join(timeout=2)
        return summarize_clocks(self.samples, self.max_mhz)


def summarize_clocks(samples, max_mhz) -> dict:
    """The line's ``clocks`` object from (sm MHz, event-reason mask, watts) samples:
    median SM clock and the union of reasons over the samples taken while the GPU
    was not idle (all samples if it always was); the idle bit itself is not listed."""
    if not samples:
        return {"sm_mhz": None, "sm_max_mhz": max_mhz, "reasons": [], "samples": 0}
    busy = [s for s in samples if not (s[1] & 0x1)] or list(samples)
    mask = 0
    for s in busy:
        mask |= s[1]
    return {
        "sm_mhz": int(statistics.median(s[0] for s in busy)),
        "sm_max_mhz": max_mhz,
        "reasons": [name for bit, name in _REASONS.items() if mask & bit and bit != 0x1],
        "samples": len(busy),
        "power_w_max": round(max(s[2] for s in busy), 1),
    }


# ---------------------------------------------------------------- GPU side --
def reduce_e2e_legs(serial_ms: float, pipe_ms: float, world: int, device) -> tuple[float, float]:
    """Max over ranks of both end-to-end legs; the pipelined one counts only if every
    rank has it (a rank that fell back passes -1).  Every rank makes the same two
    all-reduces, whatever its own result."""
    import torch
    import torch.distributed as dist

    t = torch.tensor([serial_ms, pipe_ms], dtype=torch.float64, device=device)
    if world > 1:
        t_min = t.clone()
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        dist.all_reduce(t_min, op=dist.ReduceOp.MIN)
        if float(t_min[1].item()) < 0:
            t[1] = -1.0
    return float(t[0].item()), float(t[1].item())


def exchange_row_totals(row_matrix) -> tuple[list[float], list[float]]:
    """Remote rows each rank sends and receives, from rows[src, dst] (rows a rank
    keeps for its own experts cross no link)."""
    m = row_matrix.double().clone()
    m.fill_diagonal_(0)
    return m.sum(dim=1).tolist(), m.sum(dim=0).tolist()


def zipf_gate_bias(router_w, num_experts: int, top_k: int, seed: int = 12345):
    """Per-expert gate bias whose top-k routing follows Zipf(1.0) over expert ids.

    Target shares p_e ~ 1/(e+1) (expert 0 hottest).  Starting from log p, the
    bias is refined on a 32768-token N(0,1) sample through this router by
    b_e += 0.5 * log(p_e / share_e) until the realised top-k assignment shares
    match; returns (bias, iterations, max relative share error).
    """
    import numpy as np

    p = 1.0 / np.arange(1, num_experts + 1, dtype=np.float64)
    p /= p.sum()
    rng = np.random.default_rng(seed)
    x = rng.standard_normal((32768, router_w.shape[1])).astype(np.float32)
    logits = (x @ router_w.astype(np.float32).T).astype(np.float64)
    bias = np.log(p)
    err, it = 1e9, 0
    for it in range(1, 301):
        z = logits + bias
        top = np.argpartition(-z, top_k - 1, axis=-1)[:, :top_k]
        share = np.bincount(top.reshape(-1), minlength=num_experts) / top.size
        err = float(np.max(np.abs(share - p) / p))
        if err < 0.02:
            break
        bias += 0.5 * np.log(p / np.maximum(share, 1e-6))
    return bias.astype(np.float32), it, err


def init_group(world: int, device):
    """NCCL process group over every rank of the run (None for one rank)."""
    if world <= 1:
        return None
    import torch.distributed as dist
    from datetime import timedelta

    if not dist.is_initialized():
        dist.init_process_group("nccl", device_id=device, timeout=timedelta(seconds=180))
    return dist.group.WORLD


def measure_layer(args, name: str, rank: int, world: int, device, group, steps: int,
                  warmup: int, timeline: bool = False, graph_ok: bool = True,
                  placement_override: str | None = None) -> dict:
    """MoE-layer forward (or config 4's forward) over every rank.

    Returns the measurement as a dict (the same on every rank; every rank takes
    the same collective steps): tokens/s of all ranks over ``steps`` timed
    forwards (CUDA events, max over ranks), the communication-hidden ratio from
    serialized phase times, and the device time of every exchange launch of the
    first chunk with the NVLink rate it implies.
    """
    import torch
    import torch.distributed as dist

    import moe_overlap_b200 as mo
    from moe_overlap_b200.layer import MoELayer, random_weights

    cfg = LAYER_WORKLOADS[name]
    T, H, Fd, E, K = cfg["tokens"], cfg["hidden"], cfg["ffn"], cfg["experts"], cfg["top_k"]
    bias_info, bias = None, None
    if cfg["zipf_bias"]:
        rw, _, _ = random_weights(E, H, Fd, 0.02, 0)
        bias, iters, err = zipf_gate_bias(rw.to(torch.bfloat16).float().numpy(), E, K)
        bias_info = {"fit": "per-expert, Zipf(1.0) target shares", "iterations": iters,
                     "max_rel_share_error_on_sample": round(err, 3)}

    placement_name = placement_override or args.placement
    placement = placement_name
    if placement == "balanced":
        from moe_overlap_b200.layer import balanced_placement

        # the gate's target shares: Zipf(1.0) over expert ids with the biased gate, else even
        shares = [1.0 / (e + 1) for e in range(E)] if cfg["zipf_bias"] else [1.0] * E
        placement = balanced_placement(shares, world)

    def build_layer():
        """Collective: every rank builds the layer (and its dispatcher) together."""
        lay = MoELayer(H, Fd, E, K, group=group, renormalize=cfg["renorm"],
                       router_bias=cfg["zipf_bias"], num_comm_sms=args.comm_sms,
                       micro_batch_size=args.micro_batch,
                       taper_chunks=args.taper,
                       fused_combine=None if args.combine == "auto" else args.combine == "push",
                       enable_nvtx=args.nvtx,
                       dispatch_fp8=args.dispatch_fp8,
                       solo_comm_blocks=args.solo_blocks or None,
                       expert_placement=placement,
                       gemm_streams=args.gemm_streams,
                       **({} if args.overlap_tiles == "auto"
                          else {"overlap_tiles": args.overlap_tiles == "on"}),
                       ).init_random(std=0.02, seed=0)
        if bias is not None:
            lay.router_b.copy_(torch.from_numpy(bias))
        return lay

    layer = build_layer()
    g = torch.Generator().manual_seed(1000 + rank)
    x = torch.randn(T, H, generator=g).to(torch.bfloat16).to(device)
    routing = layer.route(x)
    idx = routing[1]

    def row_matrix(sel):
        """rows[src, dst] of the assignments in ``sel`` over all ranks."""
        owner = layer._slots(sel) // layer.experts_per_rank
        rows_to = torch.bincount(owner[sel >= 0].reshape(-1), minlength=world).double()
        if world > 1:
            gathered = [torch.zeros_like(rows_to) for _ in range(world)]
            dist.all_gather(gathered, rows_to, group=group)
            return torch.stack(gathered).cpu()
        return rows_to.view(1, 1).cpu()

    mat = row_matrix(idx)
    recv_rows = mat.sum(dim=0)  # rows each rank receives, summed over senders
    remote_out, remote_in = exchange_row_totals(mat)
    busiest_rows = float(max(max(remote_out), max(remote_in)))
    first = layer.chunk_plan(T)[0]
    mat0 = row_matrix(idx[first[0]:first[1]])
    out0, in0 = exchange_row_totals(mat0)
    expert_counts = torch.bincount(idx[idx >= 0].reshape(-1), minlength=E).double()
    if world > 1:
        dist.all_reduce(expert_counts, group=group)
    realised_share = (expert_counts / expert_counts.sum()).tolist()
    flops_total = 4.0 * float(recv_rows.sum()) * H * Fd  # two GEMMs on every rank's rows

    for _ in range(max(3, warmup)):
        layer(x, routing=routing)
    torch.cuda.synchronize(device)
    mo.check_status(device, sync=True)
    # The timed forwards replay one CUDA graph per rank (device-drawn exchange epochs),
    # so host launch overhead and host stalls stay out of the device's schedule.  The
    # ranks agree on the outcome: if any rank's capture fails, every rank rebuilds the
    # layer (fresh dispatchers, host epochs) and times eager forwards instead.
    graph, graph_note = None, None
    if graph_ok:
        ok = 1
        try:
            from moe_overlap_b200.layer import ForwardGraph

            graph = ForwardGraph(layer, x, routing)
            for _ in range(3):
                graph.replay()
            torch.cuda.synchronize(device)
            mo.check_status(device, sync=True)
        except Exception as exc:  # report and time eager forwards instead
            ok = 0
            graph = None
            graph_note = f"capture failed ({type(exc).__name__}: {exc})"[:240]
            torch.cuda.synchronize(device)
        if world > 1:
            flag = torch.tensor([ok], dtype=torch.int32, device=device)
            dist.all_reduce(flag, op=dist.ReduceOp.MIN, group=group)
            if int(flag.item()) == 0 and ok:
                graph_note = "capture failed on another rank"
            ok = int(flag.item())
        if not ok:
            graph = None
            layer.close()
            layer = build_layer()
            for _ in range(max(3, warmup)):
                layer(x, routing=routing)
            torch.cuda.synchronize(device)

    sampler = ClockSampler(device)
    sampler.start()
    if world > 1:
        dist.barrier(group=group)
    torch.cuda.synchronize(device)
    marks = [torch.cuda.Event(enable_timing=True) for _ in range(steps + 1)]
    layer._device_align()  # every rank's first forward starts at the same device time
    marks[0].record()
    for i in range(steps):
        if graph is not None:
            graph.replay()
        else:
            layer(x, routing=routing)
        marks[i + 1].record()
    torch.cuda.synchronize(device)
    if world > 1:
        dist.barrier(group=group)
    clocks = sampler.stop()
    mo.check_status(device, sync=True)
    per_step = [marks[i].elapsed_time(marks[i + 1]) for i in range(steps)]
    t = torch.tensor([marks[0].elapsed_time(marks[-1]) / steps, statistics.median(per_step)],
                     dtype=torch.float64, device=device)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX, group=group)
    step_ms, median_ms = float(t[0].item()), float(t[1].item())
    graph_used = graph is not None
    # Kernels launched in the timed region: one replay launches the captured graph's
    # kernel nodes (counted by name after capture); eager steps are not counted.
    kernels_per_step = graph.kernel_counts if graph is not None else None
    gpu_launches = kernels_per_step["ours"] * steps if kernels_per_step else None
    del graph

    marks_by_rank = None
    if timeline:
        # One more forward with events at every phase boundary on the stream that
        # runs it (ms from the forward's start, per rank), behind ~1.5 ms of
        # device-side delay so the marks show the device's schedule.
        marks = []
        if world > 1:
            dist.barrier(group=group)
        torch.cuda.synchronize(device)
        torch.cuda._sleep(3_000_000)
        layer._device_align()  # the ranks' marks share a device-time origin
        layer(x, routing=routing, timeline=marks)
        torch.cuda.synchronize(device)
        mine = {n: round(marks[0][1].elapsed_time(ev), 4) for n, ev in marks[1:]}
        marks_by_rank = gather_objects(mine, world, group)

    _, phases = layer.forward_serialized(x, routing)
    comm_ms = phases["dispatch_ms"] + phases["combine_ms"]
    comp_ms = phases["experts_ms"]
    hidden = max(0.0, min(1.0, (comm_ms + comp_ms - step_ms) / comm_ms)) if comm_ms > 0 else None

    # Every exchange launch of the first chunk, run alone; per-rank device times.
    kt = gather_objects({k: round(v, 4) for k, v in layer.exchange_phase_times(x, routing).items()},
                        world, group)
    mo.check_status(device, sync=True)
    row_bytes = H * 2
    meta_bytes = K * 12 + 12  # top-k ids and weights, {source rank, token}, combine row index
    exchange = {"chunk": f"first chunk ({first[1] - first[0]} tokens per rank), "
                         f"{layer.solo_comm_blocks} blocks of 128 threads",
                "kernel_ms_per_rank": kt,
                "remote_rows_out_per_rank": [int(v) for v in out0],
                "remote_rows_in_per_rank": [int(v) for v in in0]}
    if world > 1:
        def gbps(nbytes, ms):
            return round(nbytes / (ms / 1e3) / 1e9, 1) if ms > 0 else None
        disp_ms = [sum(kt[r].get(f"dispatch_{p}", 0.0) for p in ("layout_count", "scatter", "wait"))
                   for r in range(world)]
        rates = {
            # rows this rank pushed to peers / its scatter kernel (which also waits for the peers' counts)
            "scatter_out_GBps": [gbps(out0[r] * (row_bytes + meta_bytes), kt[r].get("dispatch_scatter", 0.0))
                                 for r in range(world)],
            # rows peers pushed here / this rank's whole dispatch (start to every row landed)
            "dispatch_in_GBps": [gbps(in0[r] * (row_bytes + meta_bytes), disp_ms[r]) for r in range(world)],
            # rows this rank's tokens pulled back from peers / its pull kernel
            "pull_in_GBps": [gbps(out0[r] * row_bytes, kt[r].get("combine_pull", 0.0))
                             for r in range(world)],
        }
        busiest = max(range(world), key=lambda r: max(out0[r], in0[r]))
        exchange.update(rates)
        exchange["busiest_rank"] = busiest
        cands = [rates[k][busiest] for k in rates if rates[k][busiest] is not None]
        exchange["busiest_rank_GBps"] = max(cands) if cands else None
        exchange["nvlink_peak_GBps"] = {"nominal_per_direction": 900.0,
                                        "measured_peer_copy": PEER_COPY_GBPS}
    peak, peak_src = load_peaks()
    tflops = flops_total / (step_ms / 1e3) / 1e12
    result = {
        "metric": "MoE-layer tokens/s",
        "value": round(world * T / (step_ms / 1e3), 1),
        "unit": "tokens/s",
        "n_gpus": world,
        "steps": steps,
        "warmup": max(3, warmup),
        "ms_per_step": round(step_ms, 4),
        "ms_per_step_median": round(median_ms, 4),
        "config": {"workload": name, "description": cfg["desc"],
                   "tokens_per_rank": T, "micro_batch": args.micro_batch,
                   "chunks": [e - s for s, e in layer.chunk_plan(T)],
                   "cuda_graph": graph_used,
                   "cuda_graph_note": graph_note,
                   "kernels_per_step": kernels_per_step,
                   "combine": "push (fused into the down-projection GEMM)" if layer.fused_combine
                   else "pull",
                   "expert_placement": placement_name if placement_name != "balanced"
                   else {"balanced": placement},
                   "overlap_tiles": layer.overlap_tiles,
                   "gemm_streams": len(layer.compute_streams), "dispatch_payload":
                       "fp8 e4m3 + per-128 scales" if layer.dispatch_fp8 else "bf16",
                   "comm_sms": args.comm_sms, "gate_bias": bias_info,
                   "realised_expert_share": [round(v, 4) for v in realised_share],
                   "rows_received_per_rank": [int(v) for v in recv_rows.tolist()],
                   "parallelism": f"ep{world}"},
        "expert_gemm_tflops": round(tflops, 2),
        "expert_gemm_frac_of_peak": round(tflops / (world * peak), 4),
        "communication_hidden_ratio": None if hidden is None else round(hidden, 4),
        "serial_phase_ms": {k: round(v, 4) for k, v in phases.items()},
        "exchange": exchange,
        "nvlink": {
            "remote_rows_out_per_rank": [int(v) for v in remote_out],
            "remote_rows_in_per_rank": [int(v) for v in remote_in],
            "nvlink_floor_ms_per_exchange": round(busiest_rows * (row_bytes + meta_bytes)
                                                  / PEER_COPY_GBPS / 1e6, 4) if world > 1 else None,
        },
        "clocks": clocks,
        "gpu_launches": gpu_launches,
    }
    if marks_by_rank is not None:
        result["timeline_ms"] = {f"rank{r}": m for r, m in enumerate(marks_by_rank)}
    if world == 1 and not getattr(args, "no_extras", False):
        ref = reference_layer(layer, x, device)
        if "ms_per_step" in ref:
            ref["ours_over_reference"] = round(ref["ms_per_step"] / step_ms, 2)
        result["reference_layer"] = ref
    layer.close()
    return result


def gather_objects(obj, world: int, group) -> list:
    """``obj`` of every rank, indexed by rank (a one-item list for one rank)."""
    if world <= 1:
        return [obj]
    import torch.distributed as dist

    out = [None] * world
    dist.all_gather_object(out, obj, group=group)
    return out


def run_layer(args, rank: int, world: int, local_rank: int) -> None:
    """MoE-layer forward workloads as their own line: tokens/s, overlap, exchange rates."""
    import torch
    import torch.distributed as dist

    torch.cuda.set_device(local_rank)
    device = torch.device("cuda", local_rank)
    group = init_group(world, device)
    res = measure_layer(args, args.workload, rank, world, device, group, args.steps, args.warmup,
                        timeline=args.timeline, graph_ok=not args.no_graph)
    if rank == 0:
        line = {**res, "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
                "dtype": "bf16", "data": "synthetic (seeded N(0,1) tokens, N(0,0.02) weights)",
                "warmup": args.warmup}
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


def run_layer_train(args, rank: int, world: int, local_rank: int) -> None:
    """Config 4: tokens/s of one MoE-layer forward + backward (router, experts, exchange).

    A step is forward_autograd + backward of a fixed dout on the resident batch,
    producing dx and the router, W1 and W2 gradients (gradients are reset to None
    first, so there is no accumulation kernel).  With N ranks each runs its own
    replica of the layer on its own batch (config 4 is a one-GPU layer), so
    ``value`` is N x tokens / step.
    """
    import torch
    import torch.distributed as dist

    import moe_overlap_b200 as mo
    from moe_overlap_b200.layer import MoELayer

    cfg = LAYER_WORKLOADS[args.workload]
    torch.cuda.set_device(local_rank)
    device = torch.device("cuda", local_rank)
    init_group(world, device)
    T, H, Fd, E, K = cfg["tokens"], cfg["hidden"], cfg["ffn"], cfg["experts"], cfg["top_k"]
    layer = MoELayer(H, Fd, E, K, renormalize=cfg["renorm"], num_comm_sms=args.comm_sms,
                     micro_batch_size=T, training=True).init_random(std=0.02, seed=0)
    params = (layer.router_w, layer.w1, layer.w2)
    for p in params:
        p.requires_grad_(True)
    g = torch.Generator().manual_seed(1000 + rank)
    x_host = torch.randn(T, H, generator=g).to(torch.bfloat16)
    dout_host = (torch.randn(T, H, generator=g) * 1e-2).to(torch.bfloat16)
    x = x_host.to(device).requires_grad_(True)
    dout = dout_host.to(device)

    def step(xin, gout):
        for p in params:
            p.grad = None
        xin.grad = None
        out, probs, idx = layer.forward_autograd(xin)
        out.backward(gout)
        return probs, idx

    for _ in range(max(3, args.warmup)):
        step(x, dout)
    torch.cuda.synchronize(device)
    mo.check_status(device, sync=True)

    # Per-phase device times of one eager step (phase boundaries on the compute stream).
    def mark(name):
        ev = torch.cuda.Event(enable_timing=True)
        ev.record()
        layer.trace.append((name, ev))

    layer.trace = []
    # ~2 ms of device-side delay first: the host enqueues the step meanwhile (the step
    # has no host synchronisation), so the marks time device work, not host launches.
    torch.cuda._sleep(4_000_000)
    mark("step_start")
    step(x, dout)
    mark("router_bwd")
    torch.cuda.synchronize(device)
    marks, layer.trace = layer.trace, None
    phases = {}
    for (_, a), (name, b) in zip(marks[:-1], marks[1:]):
        phases["router_fwd" if name == "start" else name] = round(a.elapsed_time(b), 4)

    # The timed steps replay the whole step as one CUDA graph (device-drawn exchange
    # epochs), unless --no-graph; a failed capture falls back to eager steps.
    graph, graph_note = None, None
    if not args.no_graph:
        try:
            from moe_overlap_b200.layer import TrainStepGraph

            graph = TrainStepGraph(layer, x, dout)
            for _ in range(3):
                graph.replay()
            torch.cuda.synchronize(device)
            mo.check_status(device, sync=True)
        except Exception as exc:  # report and time eager steps instead
            graph = None
            graph_note = f"capture failed ({type(exc).__name__}: {exc})"[:240]
            torch.cuda.synchronize(device)

    def timed_step():
        if graph is not None:
            graph.replay()
            return graph.probs, graph.topk_idx
        return step(x, dout)

    sampler = ClockSampler(device)
    sampler.start()
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize(device)
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record()
    for _ in range(args.steps):
        probs, idx = timed_step()
    end.record()
    torch.cuda.synchronize(device)
    clocks = sampler.stop()
    mo.check_status(device, sync=True)
    step_ms = start.elapsed_time(end) / args.steps
    t = torch.tensor([step_ms], dtype=torch.float64, device=device)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    step_ms = float(t.item())

    stats = layer.stats(probs, idx)
    rows = T * K
    expert_flops = 12.0 * rows * H * Fd  # 2 forward + 2 dgrad + 2 wgrad GEMMs of 2*rows*H*F each
    tflops = expert_flops / (step_ms / 1e3) / 1e12

    e2e = None
    if not args.no_e2e:
        # Through the public API from pinned host memory: copy the batch and the
        # output gradient in, run the step, read the expert-load counts back.
        xh, gh = x_host.pin_memory(), dout_host.pin_memory()
        counts_h = torch.empty(E, dtype=torch.int64).pin_memory()
        n_e2e = max(3, args.steps // 2)
        xd = torch.empty_like(x.detach())
        gd = torch.empty_like(dout)
        torch.cuda.synchronize(device)
        s2, e2 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s2.record()
        for _ in range(n_e2e):
            if graph is not None:
                with torch.no_grad():
                    x.copy_(xh, non_blocking=True)
                    dout.copy_(gh, non_blocking=True)
                graph.replay()
                idx_e = graph.topk_idx
            else:
                xd.copy_(xh, non_blocking=True)
                gd.copy_(gh, non_blocking=True)
                xd.requires_grad_(True)
                _, idx_e = step(xd, gd)
                xd = xd.detach()
            counts_h.copy_(torch.bincount(idx_e.reshape(-1), minlength=E), non_blocking=True)
        e2.record()
        torch.cuda.synchronize(device)
        e2e_ms = s2.elapsed_time(e2) / n_e2e
        te = torch.tensor([e2e_ms], dtype=torch.float64, device=device)
        if world > 1:
            dist.all_reduce(te, op=dist.ReduceOp.MAX)
        e2e = {"value": round(world * T / (float(te.item()) / 1e3), 1), "unit": "tokens/s",
               "h2d_bytes_per_step": 2 * T * H * 2, "d2h_bytes_per_step": E * 8,
               "ms_per_step": round(float(te.item()), 4)}

    peak_burst, peak_src = load_peaks()
    peak = peak_burst
    try:
        peak = float(json.loads((REPO / "MEASURED_PEAKS.json").read_text())["bf16_tflops_sustained"])
        peak_src = "measured (MEASURED_PEAKS.json bf16_tflops_sustained)"
    except Exception:
        pass
    if rank == 0:
        line = {
            "metric": "MoE-layer tokens/s",
            "value": round(world * T / (step_ms / 1e3), 1),
            "unit": "tokens/s",
            "n_gpus": world,
            "steps": args.steps,
            "warmup": args.warmup,
            "ms_per_step": round(step_ms, 4),
            "higher_is_better": True,
            "scaling": "weak",
            "vs_baseline": None,
            "dtype": "bf16",
            "data": "synthetic (seeded N(0,1) tokens, N(0,0.02) weights)",
            "config": {"workload": args.workload, "description": cfg["desc"], "tokens_per_rank": T,
                       "comm_sms": args.comm_sms, "l2": "working set (weights 1 GiB, activations) > L2",
                       "cuda_graph": graph is not None, "cuda_graph_note": graph_note,
                       "kernels_per_step": graph.kernel_counts if graph is not None else None,
                       "parallelism": "replicas" if world > 1 else "single"},
            # kernels of this library in the timed region (graph replays only)
            "gpu_launches": (graph.kernel_counts["ours"] * args.steps
                             if graph is not None and graph.kernel_counts else None),
            "expert_load_cv": round(stats.load_cv, 4),
            "router_entropy": round(stats.entropy, 4),
            "roofline": {"bound": "tensor", "scope": "whole step, expert GEMM FLOPs only",
                         "achieved": round(tflops, 2), "peak": peak, "unit": "TFLOP/s",
                         "frac": round(tflops / peak, 4), "peak_source": peak_src, "traffic": None},
            "phase_ms": phases,
            "e2e": e2e,
            "clocks": clocks,
        }
        print(json.dumps(line), flush=True)
    layer.close()
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


class GemmRun:
    """One grouped-GEMM workload resident on this rank's GPU, timed launch by launch.

    Each timed launch is preceded by a 256 MiB write (outside its events) that
    evicts L2; the launches are timed with CUDA events on the launching stream.
    """

    def __init__(self, name: str, device, sm_count: int):
        import torch

        import moe_overlap_b200 as mo
        from tests._inputs import gemm_inputs

        self.mo, self.name, self.device, self.sm_count = mo, name, device, sm_count
        self.wl = WORKLOADS[name]
        self.counts = workload_counts(name)
        self.a_cpu, self.b_cpu, self.off_cpu = gemm_inputs(self.counts, self.wl["k"], self.wl["n"],
                                                           self.wl["dtype"], seed=0)
        self.rows = int(sum(self.counts))
        self.flops = 2.0 * self.rows * self.wl["k"] * self.wl["n"]
        self.a = self.a_cpu.to(device)
        self.b = self.b_cpu.to(device)
        self.off = self.off_cpu.to(device)
        self.counter = torch.zeros(1, dtype=torch.int32, device=device)
        self.flush = torch.empty(256 << 20, dtype=torch.uint8, device=device)
        self.stream = torch.cuda.current_stream(device)

    def step(self, a=None, off=None):
        return self.mo.persistent_grouped_gemm(self.a if a is None else a, self.b,
                                               self.off if off is None else off,
                                               num_sms=self.sm_count,
                                               use_atomic_queue=self.wl["atomic"],
                                               work_counter=self.counter)

    def timed(self, steps: int, warmup: int, world: int) -> dict:
        """Per-launch times (ms), their max-over-ranks total, and the clocks meanwhile."""
        import torch
        import torch.distributed as dist

        for _ in range(max(3, warmup)):
            self.step()
            self.flush.fill_(1)
        torch.cuda.synchronize(self.device)
        self.mo.check_status(self.device, sync=True)
        starts = [torch.cuda.Event(enable_timing=True) for _ in range(steps)]
        ends = [torch.cuda.Event(enable_timing=True) for _ in range(steps)]
        sampler = ClockSampler(self.device)
        sampler.start()
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize(self.device)
        for i in range(steps):
            self.flush.fill_(i & 0xFF)  # evict L2 between launches (outside the events)
            starts[i].record(self.stream)
            self.step()
            ends[i].record(self.stream)
        torch.cuda.synchronize(self.device)
        if world > 1:
            dist.barrier()
        clocks = sampler.stop()
        self.mo.check_status(self.device, sync=True)
        launch_ms = [s.elapsed_time(e) for s, e in zip(starts, ends)]
        total_ms = sum(launch_ms)
        if world > 1:
            t = torch.tensor([total_ms], dtype=torch.float64, device=self.device)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            total_ms = float(t.item())
        return {"launch_ms": launch_ms, "total_ms": total_ms, "clocks": clocks}

    def roofline(self, launch_ms: list) -> dict:
        peak, peak_src = load_peaks()
        achieved = self.flops / (statistics.mean(launch_ms) / 1e3) / 1e12
        return {
            "bound": "tensor",
            "achieved": round(achieved, 2),
            "peak": peak,
            "unit": UNIT,
            "frac": round(achieved / peak, 4),
            "peak_source": peak_src,
            "traffic": profiled_traffic(self.name),
            "kernel": ("moe::gg::grouped_gemm_kernel (1 SM)" if self.sm_count < 2 or
                       os.environ.get("MOE_B200_GEMM_KERNEL") == "1"
                       else "moe::gg::pair::grouped_gemm_pair_kernel (CTA pairs, TMA-store epilogue)"),
            "algorithmic_work": f"2*M*K*N = {self.flops / 1e9:.2f} GFLOP per launch "
                                f"(M={self.rows} real rows)",
            "rows_computed": rows_computed(self.counts),
        }

    def release(self) -> None:
        for name in ("a", "b", "off", "flush", "counter"):
            setattr(self, name, None)


def cublas_same_shape(run: GemmRun, steps: int, warmup: int) -> dict:
    """cuBLAS (through torch) on this workload's shape, timed like the grouped GEMM:
    a batched GEMM when every expert has the same rows (config 2), else the per-expert
    torch.matmul loop that the reference's CPU path also runs (config 3).  A library
    reference point for the roofline, not the product path."""
    import torch

    counts, k, n = run.counts, run.wl["k"], run.wl["n"]
    out = torch.empty(run.rows, n, dtype=run.a.dtype, device=run.device)
    if len(set(counts)) == 1:
        e, m = len(counts), counts[0]
        a3, c3 = run.a.view(e, m, k), out.view(e, m, n)
        fn, form = (lambda: torch.bmm(a3, run.b, out=c3)), "torch.bmm (cuBLAS batched GEMM)"
    else:
        offs = [0]
        for c in counts:
            offs.append(offs[-1] + int(c))

        def fn():
            for ex in range(len(counts)):
                if offs[ex + 1] > offs[ex]:
                    torch.matmul(run.a[offs[ex]:offs[ex + 1]], run.b[ex], out=out[offs[ex]:offs[ex + 1]])
        form = "per-expert torch.matmul loop (cuBLAS)"
    for _ in range(max(3, warmup)):
        fn()
        run.flush.fill_(1)
    evs = []
    for i in range(steps):
        run.flush.fill_(i & 0xFF)
        s0, s1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s0.record(run.stream)
        fn()
        s1.record(run.stream)
        evs.append((s0, s1))
    torch.cuda.synchronize(run.device)
    ms = statistics.mean(a.elapsed_time(b) for a, b in evs)
    return {"form": form, "tflops": round(run.flops / (ms / 1e3) / 1e12, 2), "ms_per_launch": round(ms, 5)}


# The reference checkout installed unmodified (git-ignored; it travels to the GPU box).
REF_DIR = REPO / "baseline" / "_ref"


def reference_layer(layer, x, device, steps: int = 5) -> dict:
    """The reference's own MoE layer forward on the same tokens and GPU: ``SimpleMoE``
    (src/train_moe_baseline.py:112-441) on its single-GPU path, with no exchange and
    the Triton grouped GEMMs of src/triton_grouped_gemm.py, under torch.inference_mode
    as the reference runs it.  The harness fixes what the reference leaves to its
    command line or to an A100: no shared experts, the device's SM count for the GEMMs
    (the reference derives 108 - deepep_num_sms), and this layer's gate weights and
    bias copied in so that both route alike.  Each forward is timed with CUDA events
    around the whole call, host synchronisations included, as a user of the reference
    sees it.  Context for the layer line, not the product path."""
    import torch

    if not (REF_DIR / "train_moe_baseline.py").exists():
        return {"unavailable": "the reference is not installed under baseline/_ref"}
    ref = None
    try:
        if str(REF_DIR) not in sys.path:
            sys.path.insert(0, str(REF_DIR))
        import train_moe_baseline as tmb

        H, E = layer.hidden, layer.num_experts
        ref = tmb.SimpleMoE(H, layer.ffn, E, 0, layer.top_k, ep_group=None, comm_backend="local",
                            micro_batch_size=layer.micro, expert_kernel="triton")
        ref = ref.to(device=device, dtype=torch.bfloat16)
        ref.triton_num_sms = torch.cuda.get_device_properties(device).multi_processor_count
        with torch.no_grad():
            gate = torch.nn.Linear(H, E, bias=layer.router_b is not None).to(device=device,
                                                                           dtype=torch.bfloat16)
            gate.weight.copy_(layer.router_w)
            if layer.router_b is not None:
                gate.bias.copy_(layer.router_b.to(torch.bfloat16))
            ref.router = gate
        with torch.inference_mode():
            for _ in range(2):
                ref(x)
            torch.cuda.synchronize(device)
            evs = []
            for _ in range(steps):
                s0, s1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                s0.record()
                ref(x)
                s1.record()
                evs.append((s0, s1))
            torch.cuda.synchronize(device)
        ms = statistics.mean(a.elapsed_time(b) for a, b in evs)
        return {"impl": "reference SimpleMoE forward, single-GPU path, Triton grouped GEMMs",
                "tokens_per_s": round(x.shape[0] / (ms / 1e3), 1), "ms_per_step": round(ms, 4),
                "steps": steps}
    except Exception as exc:  # reported, never timed
        return {"unavailable": f"{type(exc).__name__}: {exc}"[:240]}
    finally:
        del ref
        torch.cuda.empty_cache()


def triton_reference(run: GemmRun, steps: int, warmup: int) -> dict:
    """The reference's own GPU kernel on this workload, timed like the grouped GEMM:
    ``persistent_grouped_gemm`` of src/triton_grouped_gemm.py:326-443 (Triton, JIT-built
    on the box), with num_sms = the SM count, this workload's schedule (striped for
    config 2, the atomic queue for config 3) and the reference's default 128x128x32
    tiles.  Its output is checked against ours first.  A same-box comparison point,
    not the product path; when the module is absent or fails, the reason is reported."""
    import torch

    if not (REF_DIR / "triton_grouped_gemm.py").exists():
        return {"unavailable": "the reference is not installed under baseline/_ref"}
    try:
        if str(REF_DIR) not in sys.path:
            sys.path.insert(0, str(REF_DIR))
        import triton_grouped_gemm as ref

        ctr = torch.zeros(1, dtype=torch.int32, device=run.device)

        def fn():
            return ref.persistent_grouped_gemm(run.a, run.b, run.off, num_sms=run.sm_count,
                                               use_atomic_queue=run.wl["atomic"], work_counter=ctr)

        out = None
        for _ in range(max(3, warmup)):  # the first call JIT-compiles the kernel
            out = fn()
            run.flush.fill_(1)
        ours = run.step()
        torch.cuda.synchronize(run.device)
        diff = float((out.float() - ours.float()).abs().max().item())
        del ours
        evs = []
        for i in range(steps):
            run.flush.fill_(i & 0xFF)
            s0, s1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            s0.record(run.stream)
            fn()
            s1.record(run.stream)
            evs.append((s0, s1))
        torch.cuda.synchronize(run.device)
        ms = statistics.mean(a.elapsed_time(b) for a, b in evs)
        return {"kernel": "reference persistent_grouped_gemm (Triton), "
                          f"{'atomic' if run.wl['atomic'] else 'striped'} schedule, "
                          f"num_sms={run.sm_count}, 128x128x32 tiles",
                "tflops": round(run.flops / (ms / 1e3) / 1e12, 2), "ms_per_launch": round(ms, 5),
                "max_abs_diff_vs_ours": diff}
    except Exception as exc:  # reported, never timed
        return {"unavailable": f"{type(exc).__name__}: {exc}"[:240]}


def measure_e2e(run: GemmRun, steps: int, warmup: int, world: int) -> dict:
    """The headline metric end to end through ``persistent_grouped_gemm``.

    Every step copies A and the offsets in from pinned host memory, runs the GEMM
    and copies C back out.  The serial leg does the three on one stream; the
    pipelined leg puts copy-in, GEMM and copy-out on three streams with two input
    buffers, so step i's copy-out (PCIe device-to-host) overlaps step i+1's
    copy-in (host-to-device) and GEMM, as a caller streaming batches through the
    GEMM would run it.  The headline is the pipelined leg.
    """
    import torch
    import torch.distributed as dist

    mo, device, stream = run.mo, run.device, run.stream
    a_host = run.a_cpu.pin_memory()
    off_host = run.off_cpu.pin_memory()
    c_host = torch.empty((run.rows, run.wl["n"]), dtype=run.a_cpu.dtype).pin_memory()
    a_dev = torch.empty_like(run.a)
    off_dev = torch.empty_like(run.off)

    def e2e_step():
        a_dev.copy_(a_host, non_blocking=True)
        off_dev.copy_(off_host, non_blocking=True)
        c = run.step(a_dev, off_dev)
        c_host.copy_(c, non_blocking=True)

    s_in = torch.cuda.Stream(device)
    s_out = torch.cuda.Stream(device)
    a_bufs = [torch.empty_like(run.a) for _ in range(2)]
    off_bufs = [torch.empty_like(run.off) for _ in range(2)]
    ev_in = [torch.cuda.Event() for _ in range(2)]
    ev_gemm = [torch.cuda.Event() for _ in range(2)]
    issued = [0]

    def e2e_pipelined_step():
        i = issued[0]
        issued[0] += 1
        k = i % 2
        with torch.cuda.stream(s_in):
            if i >= 2:
                s_in.wait_event(ev_gemm[k])  # step i-2's GEMM has read a_bufs[k]
            a_bufs[k].copy_(a_host, non_blocking=True)
            off_bufs[k].copy_(off_host, non_blocking=True)
            ev_in[k].record(s_in)
        stream.wait_event(ev_in[k])
        c = run.step(a_bufs[k], off_bufs[k])
        ev_gemm[k].record(stream)
        s_out.wait_event(ev_gemm[k])
        with torch.cuda.stream(s_out):
            c_host.copy_(c, non_blocking=True)
        c.record_stream(s_out)  # C's memory is reused only after its copy-out

    def timed_leg(fn) -> float:
        for _ in range(max(3, warmup)):
            fn()
        torch.cuda.synchronize(device)
        e_start = torch.cuda.Event(enable_timing=True)
        e_end = torch.cuda.Event(enable_timing=True)
        e_start.record(stream)
        s_in.wait_stream(stream)
        for _ in range(steps):
            fn()
        stream.wait_stream(s_in)
        stream.wait_stream(s_out)
        e_end.record(stream)
        torch.cuda.synchronize(device)
        return e_start.elapsed_time(e_end)

    if world > 1:
        dist.barrier()
    serial_ms = timed_leg(e2e_step)
    want_c = c_host.clone()
    c_host.zero_()
    pipe_ms = -1.0
    if world > 1:
        dist.barrier()
    try:
        pipe_ms = timed_leg(e2e_pipelined_step)
        if not torch.equal(c_host, want_c):
            raise RuntimeError("pipelined result differs from the serial one")
    except RuntimeError as exc:  # keep the serial figure, say why
        print(f"bench: pipelined end-to-end leg not used: {exc}", file=sys.stderr, flush=True)
        pipe_ms = -1.0
    serial_ms, pipe_ms = reduce_e2e_legs(serial_ms, pipe_ms, world, device)
    mo.check_status(device, sync=True)
    e2e_ms = pipe_ms if pipe_ms > 0 else serial_ms
    return {
        "value": round(world * run.flops * steps / (e2e_ms / 1e3) / 1e12, 3),
        "unit": UNIT,
        "h2d_bytes_per_step": a_host.numel() * a_host.element_size()
        + off_host.numel() * off_host.element_size(),
        "d2h_bytes_per_step": c_host.numel() * c_host.element_size(),
        "ms_per_step": round(e2e_ms / steps, 4),
        "pipelined": pipe_ms > 0,
        "serial_ms_per_step": round(serial_ms / steps, 4),
    }


def main() -> None:
    args = parse_args()
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference":
        run_reference(args, rank)
        return
    if args.workload == "layer_train":
        run_layer_train(args, rank, world, local_rank)
        return
    if args.workload in LAYER_WORKLOADS:
        run_layer(args, rank, world, local_rank)
        return

    import torch
    import torch.distributed as dist

    if not torch.cuda.is_available():
        raise RuntimeError("bench.py needs a CUDA device")
    torch.cuda.set_device(local_rank)
    device = torch.device("cuda", local_rank)
    group = init_group(world, device)
    sm_count = torch.cuda.get_device_properties(device).multi_processor_count

    run = GemmRun(args.workload, device, sm_count)
    res = run.timed(args.steps, args.warmup, world)
    value = world * run.flops * args.steps / (res["total_ms"] / 1e3) / 1e12
    e2e = None if args.no_e2e else measure_e2e(run, args.steps, args.warmup, world)
    roofline = run.roofline(res["launch_ms"])
    lib_ref = cublas_same_shape(run, args.steps, args.warmup)
    lib_ref["ours_over_cublas"] = round(roofline["achieved"] / lib_ref["tflops"], 4)
    roofline["cublas_same_shape"] = lib_ref
    # The reference's Triton kernel beside ours on one GPU (a per-GPU comparison; at N > 1
    # every rank would JIT-build it into the same cache at once).
    if not args.no_extras and world == 1:
        tri = triton_reference(run, args.steps, args.warmup)
        if "tflops" in tri:
            tri["ours_over_triton"] = round(roofline["achieved"] / tri["tflops"], 4)
        roofline["triton_reference"] = tri
    run.release()
    torch.cuda.empty_cache()

    extras = {}
    if args.workload == "gemm_cfg2" and not args.no_extras:
        # BASELINE config 3 (the skewed config the north-star target names), timed alike.
        r3 = GemmRun("gemm_cfg3", device, sm_count)
        t3 = r3.timed(args.steps, args.warmup, world)
        extras["gemm_cfg3"] = {
            "value": round(world * r3.flops * args.steps / (t3["total_ms"] / 1e3) / 1e12, 3),
            "unit": UNIT,
            "ms_per_step": round(t3["total_ms"] / args.steps, 5),
            "steps": args.steps,
            "config": gemm_config("gemm_cfg3", sm_count, world),
            "roofline": r3.roofline(t3["launch_ms"]),
            "clocks": t3["clocks"],
        }
        lib3 = cublas_same_shape(r3, args.steps, args.warmup)
        lib3["ours_over_cublas"] = round(extras["gemm_cfg3"]["roofline"]["achieved"] / lib3["tflops"], 4)
        extras["gemm_cfg3"]["roofline"]["cublas_same_shape"] = lib3
        if world == 1:
            tri3 = triton_reference(r3, args.steps, args.warmup)
            if "tflops" in tri3:
                tri3["ours_over_triton"] = round(extras["gemm_cfg3"]["roofline"]["achieved"]
                                                 / tri3["tflops"], 4)
            extras["gemm_cfg3"]["roofline"]["triton_reference"] = tri3
        r3.release()
        del r3
        torch.cuda.empty_cache()
        # the expert-parallel layer over every rank of this run.
        ep = measure_layer(args, "ep_layer", rank, world, device, group,
                           steps=min(args.steps, 20), warmup=args.warmup)
        for key in ("metric",):
            ep.pop(key, None)
        extras["ep_layer"] = ep
        torch.cuda.empty_cache()
        if world > 1:
            # The same layer with its experts placed by expected load instead of the
            # reference's contiguous blocks (the Zipf gate puts the hot experts on rank 0).
            bal = measure_layer(args, "ep_layer", rank, world, device, group,
                                steps=min(args.steps, 20), warmup=args.warmup,
                                placement_override="balanced")
            extras["ep_layer_balanced_placement"] = {
                k: bal[k] for k in ("value", "unit", "ms_per_step", "ms_per_step_median",
                                    "communication_hidden_ratio", "serial_phase_ms",
                                    "expert_gemm_tflops", "gpu_launches")}
            extras["ep_layer_balanced_placement"]["config"] = {
                k: bal["config"][k] for k in ("expert_placement", "rows_received_per_rank",
                                              "cuda_graph", "kernels_per_step", "parallelism")}
            torch.cuda.empty_cache()

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        cpu = cpu_baseline(args.workload)

    if rank == 0:
        line = {
            "metric": METRIC,
            "value": round(value, 3),
            "unit": UNIT,
            "n_gpus": world,
            "steps": args.steps,
            "warmup": args.warmup,
            "ms_per_step": round(res["total_ms"] / args.steps, 5),
            "higher_is_better": True,
            "scaling": "weak",
            "vs_baseline": None,
            "dtype": run.wl["dtype"],
            "data": "synthetic (seeded N(0,1) activations, N(0,0.02) weights; generated on CPU)",
            "config": gemm_config(args.workload, sm_count, world),
            "roofline": roofline,
            "cpu_baseline": cpu,
            "e2e": e2e,
            "clocks": res["clocks"],
            "gpu_launches": args.steps,
            **extras,
        }
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
