"""Routed MoE layer on B200: router -> dispatch -> grouped GEMMs -> weighted combine.

The forward of SimpleMoE's routed path (src/train_moe_baseline.py:315-441)
built from this package's kernels, with none of the reference's per-call host
work:
  * expert weights stay in nn.Linear layout ([E_local, F, H] and [E_local, H, F])
    and are fed to the grouped GEMM as K-major views (the reference re-stacks and
    transposes them on every call, :187-191);
  * dispatch writes rows straight into each owner's expert-ordered receive slot
    and produces expert_offsets on the device, so there is no sort, bincount or
    .item() (:219-234);
  * GELU is fused into the up-projection's epilogue (:243), the down-projection
    writes into the exchange buffer, and the combine applies the top-k weights
    while it reduces (:394-399 + deep_ep_comm.combine);
  * the router's softmax / bias / top-k / renormalisation is one kernel
    (router.router_topk) after the gate matmul (:316-318);
  * chunks of ``micro_batch_size`` tokens pipeline like the reference's loop
    (:349-441): the next chunk's dispatch runs on the exchange stream while the
    current chunk's GEMMs run on the compute stream, on the same SMs (the
    exchange blocks are sized to run beside the persistent GEMM CTAs).
World size 1 (no process group) runs the same kernels with a local exchange.
Training: forward_autograd / RoutedExperts (backward on the same kernels), and
TrainStepGraph to replay a whole training step as one CUDA graph.
"""
from __future__ import annotations

import contextlib
from dataclasses import dataclass
from typing import Optional

import torch
import torch.distributed as dist

from .deep_ep_comm import DeepEPDispatcher
from .fp8 import dequantize_fp8, quantize_fp8
from .gemm import grouped_gemm, grouped_gemm_wgrad
from .router import router_topk

# Expert segments of a training dispatch are padded to this many rows so the
# weight-gradient GEMM's 64-row k-blocks never straddle two experts.
TRAIN_ALIGNMENT = 64


@contextlib.contextmanager
def nvtx_range(name: str, enabled: bool):
    """An NVTX range around host-side enqueueing when ``enabled`` (and CUDA is
    present), as the reference's SimpleMoE marks its chunks with --enable-nvtx
    (src/train_moe_baseline.py:74-83)."""
    if enabled and torch.cuda.is_available():
        torch.cuda.nvtx.range_push(name)
        try:
            yield
        finally:
            torch.cuda.nvtx.range_pop()
    else:
        yield


@dataclass
class RouterStats:
    entropy: float
    load_std: float
    load_cv: float


def expert_placement_order(num_experts: int, world: int, placement="contiguous") -> list:
    """Global expert id held by each placement slot; rank r owns slots
    [r * E/W, (r + 1) * E/W), in that order, as its local experts.

    ``"contiguous"`` is the reference's sharding (rank r holds experts r*E/W ..,
    src/train_moe_baseline.py:136-137).  ``"strided"`` deals the experts out like
    cards (rank r holds r, r + W, r + 2W, ...), which spreads a skew that follows
    the expert ids (e.g. a Zipf gate with expert 0 hottest) over the ranks.  A
    sequence gives the order itself (a permutation of the expert ids).
    """
    if num_experts % world != 0:
        raise ValueError(f"num_experts ({num_experts}) must be divisible by world_size ({world})")
    per = num_experts // world
    if isinstance(placement, str):
        if placement == "contiguous":
            return list(range(num_experts))
        if placement == "strided":
            return [le * world + r for r in range(world) for le in range(per)]
        raise ValueError(f"unknown expert placement {placement!r}")
    order = [int(e) for e in placement]
    if sorted(order) != list(range(num_experts)):
        raise ValueError("an expert placement must be a permutation of the expert ids")
    return order


def balanced_placement(loads, world: int) -> list:
    """A placement order (for ``expert_placement``) that evens out the expected rows
    per rank: experts taken from the heaviest ``loads[e]`` down, each given to the
    rank with the least load so far among those with a free slot (longest
    processing time first, E/W experts per rank).  Ties go to the lower rank, so
    the result is deterministic and the same on every rank."""
    loads = [float(v) for v in loads]
    num_experts = len(loads)
    if world < 1 or num_experts % world != 0:
        raise ValueError(f"num_experts ({num_experts}) must be divisible by world_size ({world})")
    per = num_experts // world
    held = [[] for _ in range(world)]
    total = [0.0] * world
    for e in sorted(range(num_experts), key=lambda i: (-loads[i], i)):
        r = min((r for r in range(world) if len(held[r]) < per), key=lambda r: (total[r], r))
        held[r].append(e)
        total[r] += loads[e]
    return [e for r in range(world) for e in held[r]]


def random_weights(num_experts: int, hidden: int, ffn: int, std: float = 0.02, seed: int = 0):
    """(router [E, H], w1 [E, F, H], w2 [E, H, F]) fp32 CPU tensors, N(0, std), seeded."""
    g = torch.Generator().manual_seed(seed)
    rw = torch.randn(num_experts, hidden, generator=g) * std
    w1 = torch.randn(num_experts, ffn, hidden, generator=g) * std
    w2 = torch.randn(num_experts, hidden, ffn, generator=g) * std
    return rw, w1, w2


class MoELayer:
    """Expert-parallel routed MoE layer.

    The grouped GEMMs use the atomic tile queue by default: they share the SMs
    with the exchange kernels, and a CTA pair slowed by an exchange block beside
    it then simply takes fewer tiles instead of delaying a fixed striped share.
    ``num_comm_sms`` is the exchange kernels' grid (128-thread blocks) for the
    phases that overlap a GEMM; the first dispatch, the last combine and the
    training path use four blocks per SM.  ``fused_combine`` selects the
    GEMM-fused combine push (off by default; it measured even with the pull).
    """

    def __init__(self, hidden_size: int, ffn_size: int, num_experts: int, top_k: int, *,
                 group: Optional[dist.ProcessGroup] = None, renormalize: bool = False,
                 router_bias: bool = False, num_comm_sms: int = 148,
                 micro_batch_size: int = 4096, use_atomic_queue: bool = True,
                 max_recv_rows: Optional[int] = None, training: bool = False,
                 taper_chunks: bool = False, fused_combine: Optional[bool] = None,
                 enable_nvtx: bool = False, dispatch_fp8: bool = False,
                 overlap_tiles: bool = False, solo_comm_blocks: Optional[int] = None,
                 expert_placement="contiguous", gemm_streams: int = 2):
        self.hidden, self.ffn, self.num_experts, self.top_k = hidden_size, ffn_size, num_experts, top_k
        # NVTX ranges named as the reference's (deepep_dispatch_chunk_i,
        # expert_compute_chunk_i, deepep_combine_chunk_i; train_moe_baseline.py:364-413)
        self.enable_nvtx = enable_nvtx
        self.group = group
        self.world = group.size() if group is not None else 1
        self.rank = group.rank() if group is not None else 0
        if num_experts % self.world != 0:
            raise ValueError(f"num_routed_experts ({num_experts}) must be divisible by world_size ({self.world})")
        self.experts_per_rank = num_experts // self.world
        # Which global experts this rank holds (expert_placement_order); the exchange
        # sees placement slots, so a non-contiguous placement is a relabelling of the
        # router's ids before each dispatch, and the weights follow it.
        order = expert_placement_order(num_experts, self.world, expert_placement)
        per = self.experts_per_rank
        self.local_experts = order[self.rank * per:(self.rank + 1) * per]
        self._slot_of_expert = None
        if order != list(range(num_experts)):
            slot_of = [0] * num_experts
            for slot, e in enumerate(order):
                slot_of[e] = slot
            self._slot_of_expert = torch.tensor(slot_of, dtype=torch.int64,
                                                device=torch.device("cuda", torch.cuda.current_device()))
        self.renormalize = renormalize
        self.micro = max(1, int(micro_batch_size))
        self.taper = taper_chunks
        # The GEMM-fused combine push (expert_gemm_push + combine_pushed) is off by
        # default: with TMA bulk stores into the source ranks it ties the separate
        # pull combine (config 5 on 2 B200s, per-step medians: 1.596 / 1.600 ms
        # against 1.592 / 1.590 ms), and its longer GEMM hides the same exposure.
        self.fused_combine = bool(fused_combine) if fused_combine is not None else False
        self.use_atomic = use_atomic_queue
        # FP8 dispatch payload (forward only): each chunk is quantised per 128
        # columns (e4m3 + float scales, DeepEP's FP8 format), dispatched in that form
        # and dequantised to bf16 on the owner before its up-projection.
        if dispatch_fp8 and (training or hidden_size % 128 != 0):
            raise ValueError("dispatch_fp8 needs the forward path and a hidden size that is a "
                             "multiple of 128")
        self.dispatch_fp8 = bool(dispatch_fp8)
        # Tile-granular overlap of each dispatch with its up-projection: expert-ordered
        # dispatch, and GEMM1 (DeepEPDispatcher.expert_gemm) enqueued as soon as this
        # rank's rows are sent; its tiles start expert by expert as their rows land.
        if overlap_tiles and (training or dispatch_fp8):
            raise ValueError("overlap_tiles is a forward option for bf16 dispatches")
        self.overlap_tiles = bool(overlap_tiles)
        self.device = torch.device("cuda", torch.cuda.current_device())
        dev, bf16 = self.device, torch.bfloat16
        self.router_w = torch.zeros(num_experts, hidden_size, dtype=bf16, device=dev)
        self.router_b = torch.zeros(num_experts, dtype=torch.float32, device=dev) if router_bias else None
        self.w1 = torch.zeros(self.experts_per_rank, ffn_size, hidden_size, dtype=bf16, device=dev)
        self.w2 = torch.zeros(self.experts_per_rank, hidden_size, ffn_size, dtype=bf16, device=dev)
        if training and max_recv_rows is None:
            # worst case of one dispatch (every rank sends all its assignments here)
            # plus the alignment padding of every local expert
            max_recv_rows = (self.world * self.micro * min(top_k, self.experts_per_rank)
                             + self.experts_per_rank * TRAIN_ALIGNMENT)
        self.dispatcher = DeepEPDispatcher(group, hidden_size, num_experts, num_sms=num_comm_sms,
                                           max_tokens_per_rank=self.micro, max_top_k=top_k,
                                           max_recv_rows=max_recv_rows, exact_size=False)
        # The forward's chunks alternate over ``gemm_streams`` compute streams (1 or 2),
        # each with its own GEMM1 output and work counter, so the next chunk's GEMM1
        # can take the SMs that the last wave of this chunk's GEMM2 leaves idle.
        if gemm_streams not in (1, 2):
            raise ValueError("gemm_streams must be 1 or 2")
        if training:
            gemm_streams = 1  # the training step is one chunk
        self.compute_streams = [torch.cuda.Stream(dev) for _ in range(gemm_streams)]
        self.compute_stream = self.compute_streams[0]
        self.gemm_sms = torch.cuda.get_device_properties(dev).multi_processor_count
        # Exchange blocks when nothing runs beside them (the training path waits for
        # each exchange phase): four 128-thread blocks per SM.
        self.solo_comm_blocks = int(solo_comm_blocks) if solo_comm_blocks else 4 * self.gemm_sms
        self.hs = [torch.empty(self.dispatcher.max_recv_rows, ffn_size, dtype=bf16, device=dev)
                   for _ in range(gemm_streams)]
        self.counters = [torch.zeros(1, dtype=torch.int32, device=dev) for _ in range(gemm_streams)]
        self.h, self.counter = self.hs[0], self.counters[0]
        # When a list, the training path appends (phase, event) pairs recorded on
        # the compute stream at each phase boundary (for per-phase device times).
        self.trace: Optional[list] = None

    # ----------------------------------------------------------------- weights --
    def init_random(self, std: float = 0.02, seed: int = 0) -> "MoELayer":
        """N(0, std) weights drawn on the CPU: every rank draws all experts and keeps its own."""
        rw, w1, w2 = random_weights(self.num_experts, self.hidden, self.ffn, std, seed)
        mine = torch.tensor(self.local_experts, dtype=torch.int64)
        self.router_w.copy_(rw.to(torch.bfloat16))
        self.w1.copy_(w1[mine].to(torch.bfloat16))
        self.w2.copy_(w2[mine].to(torch.bfloat16))
        return self

    def load_reference_state_dict(self, sd: dict) -> "MoELayer":
        """Weights from a single-process SimpleMoE state_dict (global expert ids)."""
        self.router_w.copy_(sd["router.weight"].to(torch.bfloat16))
        for le, e in enumerate(self.local_experts):
            self.w1[le].copy_(sd[f"routed_experts.{e}.w1.weight"].to(torch.bfloat16))
            self.w2[le].copy_(sd[f"routed_experts.{e}.w2.weight"].to(torch.bfloat16))
        return self

    # ----------------------------------------------------------------- forward --
    def route(self, x: torch.Tensor):
        """softmax router and top-k (src/train_moe_baseline.py:316-318); float32 weights.

        The gate's linear layer is one bf16 matmul (bf16 logits, as under the
        reference's autocast); softmax, bias, top-k and renormalisation are one
        kernel (router.router_topk)."""
        with torch.no_grad():
            logits = torch.matmul(x.to(torch.bfloat16), self.router_w.detach().t())
            return router_topk(logits, self.top_k, bias=self.router_b, renormalize=self.renormalize)

    def _slots(self, idx: torch.Tensor) -> torch.Tensor:
        """The router's global expert ids as placement slots (unchanged for the
        reference's contiguous placement; -1 stays -1)."""
        if self._slot_of_expert is None:
            return idx
        return torch.where(idx >= 0, self._slot_of_expert[idx.clamp_min(0)], idx)

    def _dispatch(self, xs, idx, w, **kw):
        """One chunk's dispatch: bf16 rows, or with ``dispatch_fp8`` the chunk quantised
        to e4m3 + per-128 scales on the current stream and dispatched in that form."""
        idx = self._slots(idx)
        if not self.dispatch_fp8:
            return self.dispatcher.dispatch(xs, idx, w, ordered=self.overlap_tiles, **kw)
        kw.pop("timeline", None)
        return self.dispatcher.dispatch_fp8(quantize_fp8(xs), idx, w, **kw)

    def _experts(self, res, buf: int = 0) -> Optional[torch.Tensor]:
        """GEMM1 (+GELU) and GEMM2 on the current stream, through GEMM1 output and
        work counter ``buf`` (the compute stream's own).

        With ``fused_combine`` GEMM2's epilogue pushes each row straight to its
        source rank (DeepEPDispatcher.expert_gemm_push) and None is returned;
        otherwise the expert-output rows are written locally and returned.
        An FP8 receive payload is first dequantised into the slot's expert-output
        rows, which GEMM1 reads before GEMM2 overwrites them."""
        h = self.hs[buf]
        kw = dict(num_sms=self.gemm_sms, use_atomic_queue=self.use_atomic, work_counter=self.counters[buf])
        a = res.recv_x
        if isinstance(a, tuple):
            buf = self.dispatcher.expert_out_buffer(res.handle)
            a = dequantize_fp8(a[0], a[1], out=buf[:a[0].shape[0]], rows=res.expert_offsets[-1:])
        if getattr(res.handle, "ordered", False):
            self.dispatcher.expert_gemm(res.handle, self.w1.transpose(1, 2), h,
                                        activation="gelu", **kw)
        else:
            grouped_gemm(a, self.w1.transpose(1, 2), res.expert_offsets, out=h,
                         activation="gelu", **kw)
        if self.fused_combine:
            self.dispatcher.expert_gemm_push(h, self.w2.transpose(1, 2), res.handle, **kw)
            return None
        y = self.dispatcher.expert_out_buffer(res.handle)
        grouped_gemm(h, self.w2.transpose(1, 2), res.expert_offsets, out=y, **kw)
        return y

    def _combine(self, y, handle, **kw):
        if y is None:
            return self.dispatcher.combine_pushed(handle, weighted=True, **kw)
        return self.dispatcher.combine(y, handle, weighted=True, **kw)

    def chunk_plan(self, t_total: int) -> list:
        """Token ranges of the pipelined chunks (each at most micro_batch_size tokens).

        Only the first chunk's dispatch and the last chunk's combine have no
        expert GEMM to hide behind, so with ``taper_chunks`` (when the batch spans
        several chunks) those two chunks are a quarter of micro_batch_size and the
        tokens between them are split evenly.  Off by default: on 2 B200s with
        BASELINE config 5 the smaller GEMMs cost more (1.77 vs 1.66 ms per step)
        than the exposed exchange they save.
        """
        m = self.micro
        if t_total <= m:
            return [(0, t_total)]
        edge = max(1, m // 4) if self.taper else m
        if not self.taper or t_total <= 2 * edge:
            return [(s, min(s + m, t_total)) for s in range(0, t_total, m)]
        mid = t_total - 2 * edge
        n_mid = -(-mid // m)
        bounds = [0, edge] + [edge + (mid * (i + 1)) // n_mid for i in range(n_mid)] + [t_total]
        return list(zip(bounds[:-1], bounds[1:]))

    @staticmethod
    def _timeline_mark(timeline, name: str, stream) -> None:
        if timeline is not None:
            ev = torch.cuda.Event(enable_timing=True)
            ev.record(stream)
            timeline.append((name, ev))

    def forward(self, x: torch.Tensor, return_stats: bool = False, routing=None,
                timeline: Optional[list] = None):
        """Returns (out [T, H] bf16, RouterStats or None).  ``routing`` = (probs, idx, w) to reuse.

        ``timeline`` (a list) receives (name, CUDA event) pairs recorded on the
        stream that runs each phase: the end of each chunk's dispatch and combine on
        the exchange stream, the start and end of its GEMMs on the compute stream.
        """
        x = x.to(torch.bfloat16).contiguous()
        probs, idx, w = routing if routing is not None else self.route(x)
        t_total = x.shape[0]
        out = torch.empty_like(x)
        chunks = self.chunk_plan(t_total)
        disp = self.dispatcher
        cur_stream = torch.cuda.current_stream(self.device)
        self._timeline_mark(timeline, "start", cur_stream)
        # The first dispatch and the last combine have no GEMM beside them: they get
        # the solo grid; the others run one block per SM beside the GEMMs.
        nv = self.enable_nvtx
        with nvtx_range("deepep_dispatch_chunk_0", nv):
            cur = self._dispatch(x[chunks[0][0]:chunks[0][1]], idx[chunks[0][0]:chunks[0][1]],
                                 w[chunks[0][0]:chunks[0][1]], pad_rows=False,
                                 num_sms=self.solo_comm_blocks)
        self._timeline_mark(timeline, "dispatch0_end", disp.comm_stream)
        for i, (s, e) in enumerate(chunks):
            # Enqueue this chunk's GEMMs before the next chunk's dispatch: the GPU
            # starts them as soon as this chunk's rows have landed, and the host
            # time spent enqueuing the next dispatch overlaps them.
            buf = i % len(self.compute_streams)
            cs = self.compute_streams[buf]
            with torch.cuda.stream(cs), nvtx_range(f"expert_compute_chunk_{i}", nv):
                # An ordered dispatch's GEMM may start once this rank's rows are sent.
                cur.extra.get("scatter_event", cur.event).current_stream_wait()
                self._timeline_mark(timeline, f"gemm{i}_start", cs)
                y = self._experts(cur, buf)
                self._timeline_mark(timeline, f"gemm{i}_end", cs)
                done = torch.cuda.Event()
                done.record(cs)
            nxt = None
            if i + 1 < len(chunks):
                ns, ne = chunks[i + 1]
                with nvtx_range(f"deepep_dispatch_chunk_{i + 1}", nv):
                    nxt = self._dispatch(x[ns:ne], idx[ns:ne], w[ns:ne], pad_rows=False)
                self._timeline_mark(timeline, f"dispatch{i + 1}_end", disp.comm_stream)
            last = i + 1 == len(chunks)
            with nvtx_range(f"deepep_combine_chunk_{i}", nv):
                self._combine(y, cur.handle, previous_event=done, out=out[s:e],
                              num_sms=self.solo_comm_blocks if last else None)
            self._timeline_mark(timeline, f"combine{i}_end", disp.comm_stream)
            cur = nxt
        torch.cuda.current_stream(self.device).wait_stream(disp.comm_stream)
        self._timeline_mark(timeline, "end", cur_stream)
        stats = self.stats(probs, idx) if return_stats else None
        return out, stats

    __call__ = forward

    def forward_serialized(self, x: torch.Tensor, routing,
                           host_cover_cycles: int = 2_000_000) -> tuple[torch.Tensor, dict]:
        """The same forward with every phase run alone, for overlap accounting.

        Each chunk's dispatch, expert GEMMs and combine run one after another
        with a device synchronisation (and, across ranks, a barrier) between
        phases; returns the output and the summed device time of each phase in
        ms (max over ranks), i.e. the serial times that the overlapped forward
        hides behind each other.  Each phase is enqueued behind a device-side
        delay of ``host_cover_cycles`` SM cycles (~1 ms), started before its
        events, so the host's enqueueing of the phase (argument checks and
        several launches) happens while the GPU is busy and the events time the
        phase's device work only, as it runs inside the pipelined forward; a
        one-element all-reduce after the delay lines the ranks up on the device, so
        a phase's time does not include another rank's late start.
        """
        x = x.to(torch.bfloat16).contiguous()
        _, idx, w = routing
        out = torch.empty_like(x)
        t_total = x.shape[0]
        chunks = self.chunk_plan(t_total)
        times = {"dispatch_ms": 0.0, "experts_ms": 0.0, "combine_ms": 0.0}
        disp = self.dispatcher

        def timed(key, fn):
            self._sync_all()
            start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            if host_cover_cycles > 0:
                torch.cuda._sleep(int(host_cover_cycles))
            self._device_align()
            start.record()
            r = fn()
            torch.cuda.current_stream(self.device).wait_stream(disp.comm_stream)
            end.record()
            self._sync_all()
            times[key] += start.elapsed_time(end)
            return r

        for s, e in chunks:
            res = timed("dispatch_ms", lambda: self._dispatch(x[s:e], idx[s:e], w[s:e], pad_rows=False))
            res.event.current_stream_wait()
            y = timed("experts_ms", lambda: self._experts(res))
            timed("combine_ms", lambda: self._combine(y, res.handle, out=out[s:e]))
        if self.world > 1:
            t = torch.tensor([times[k] for k in sorted(times)], dtype=torch.float64, device=self.device)
            dist.all_reduce(t, op=dist.ReduceOp.MAX, group=self.group)
            times = dict(zip(sorted(times), t.tolist()))
        return out, times

    def exchange_phase_times(self, x: torch.Tensor, routing,
                             host_cover_cycles: int = 2_000_000) -> dict:
        """Device time (ms) of each exchange launch of the first chunk, run alone.

        The first chunk's dispatch (layout + count push, scatter, wait for every
        peer's rows) and, after its expert GEMMs, its combine (ready flag, pull +
        reduce) run with a device synchronisation and, across ranks, a barrier
        before each, behind a device-side delay of ``host_cover_cycles`` SM cycles
        so the host's enqueueing is not timed, and a device-side all-reduce that
        lines the ranks up.  Both use the grid of the forward's
        unoverlapped phases (four blocks per SM).  Returns this rank's times:
        ``dispatch_layout_count``, ``dispatch_scatter``, ``dispatch_wait``,
        ``combine_ready``, ``combine_pull``.  The scatter includes the wait for
        every peer's counts, and the dispatch's wait the arrival of the peers' rows.
        """
        x = x.to(torch.bfloat16).contiguous()
        _, idx, w = routing
        s, e = self.chunk_plan(x.shape[0])[0]
        disp = self.dispatcher
        marks_d, marks_c = [], []
        self._sync_all()
        if host_cover_cycles > 0:
            torch.cuda._sleep(int(host_cover_cycles))
        self._device_align()
        res = self._dispatch(x[s:e], idx[s:e], w[s:e], pad_rows=False,
                             num_sms=self.solo_comm_blocks, timeline=marks_d)
        res.event.current_stream_wait()
        y = self._experts(res)
        self._sync_all()
        if host_cover_cycles > 0:
            torch.cuda._sleep(int(host_cover_cycles))
        self._device_align()
        out = torch.empty(e - s, self.hidden, dtype=torch.bfloat16, device=self.device)
        if y is None:  # fused combine push: the transfer ran inside the GEMM
            _, ev = self._combine(None, res.handle, out=out, num_sms=self.solo_comm_blocks)
        else:
            _, ev = disp.combine(y, res.handle, weighted=True, out=out,
                                 num_sms=self.solo_comm_blocks, timeline=marks_c)
        ev.current_stream_wait()
        self._sync_all()
        times = {}
        for marks, prefix in ((marks_d, "dispatch_"), (marks_c, "combine_")):
            for (_, a), (name, b) in zip(marks[:-1], marks[1:]):
                times[prefix + name] = a.elapsed_time(b)
        return times

    def _device_align(self) -> None:
        """A one-element all-reduce on the current stream: every rank's work enqueued
        after it starts when the slowest rank has reached it, so timed phases begin at
        the same device time on every GPU instead of one host barrier's skew apart."""
        if self.world > 1:
            if getattr(self, "_align_buf", None) is None:
                self._align_buf = torch.zeros(1, dtype=torch.float32, device=self.device)
            dist.all_reduce(self._align_buf, group=self.group)

    def _sync_all(self) -> None:
        torch.cuda.synchronize(self.device)
        if self.world > 1:
            dist.barrier(group=self.group)

    def stats(self, probs: torch.Tensor, idx: torch.Tensor) -> RouterStats:
        """Router entropy and expert-load spread (src/train_moe_baseline.py:450-461)."""
        counts = torch.bincount(idx.reshape(-1), minlength=self.num_experts).float()
        if self.world > 1:
            dist.all_reduce(counts, group=self.group)
        mean = counts.mean().clamp_min(1e-6)
        entropy = (-probs * probs.clamp_min(1e-9).log()).sum(dim=-1).mean()
        return RouterStats(float(entropy.detach()), float(counts.std()), float(counts.std() / mean))

    # ---------------------------------------------------------------- training --
    def forward_autograd(self, x: torch.Tensor):
        """Differentiable forward: returns (out, probs, topk_idx).

        The gate's linear layer runs in torch autograd, softmax / top-k /
        renormalisation in router.RouterTopK (forward and backward kernels); the routed experts run on this package's kernels through
        RoutedExperts (dispatch, GEMM1+GELU saving gelu'(a) from the same erf,
        GEMM2, weighted combine; backward: top-k weight gradient, weighted
        dispatch of the output gradient, dgrad GEMMs with the saved gelu'
        multiplied in, combine, weight-gradient GEMMs).  ``router_w``, ``w1`` and ``w2`` receive ``.grad`` when they
        require it.  The whole batch is one chunk (micro_batch_size must cover it),
        and nothing runs beside the exchange kernels in this path (each phase waits
        for the one before), so they run on the caller's stream (no stream switch)
        with four blocks per SM; only the backward's combine of dx runs on the
        exchange stream, beside the weight-gradient GEMMs.
        """
        logits = torch.matmul(x.to(torch.bfloat16), self.router_w.t())
        probs, idx, w = router_topk(logits, self.top_k, bias=self.router_b,
                                    renormalize=self.renormalize)
        out = RoutedExperts.apply(x, w, self.w1, self.w2, idx, self)
        return out, probs, idx

    def _mark(self, phase: str) -> None:
        if self.trace is not None:
            ev = torch.cuda.Event(enable_timing=True)
            ev.record()
            self.trace.append((phase, ev))

    def _train_forward(self, x: torch.Tensor, idx: torch.Tensor, w: torch.Tensor):
        disp = self.dispatcher
        self._mark("start")
        if x.shape[0] > self.micro:
            raise ValueError("training forward runs the batch as one chunk: raise micro_batch_size")
        x = x.to(torch.bfloat16).contiguous()
        res = disp.dispatch(x, self._slots(idx), w.float(), exact_size=False, pad_rows=False,
                            inline=True, expert_alignment=TRAIN_ALIGNMENT,
                            num_sms=self.solo_comm_blocks)
        res.event.current_stream_wait()
        self._mark("fwd_dispatch")
        rows = res.recv_x.shape[0]
        pre = torch.empty(rows, self.ffn, dtype=torch.bfloat16, device=self.device)  # gelu'(a)
        h = torch.empty_like(pre)
        kw = dict(num_sms=self.gemm_sms, use_atomic_queue=self.use_atomic, work_counter=self.counter)
        # h = GELU(a) and, from the same erf, gelu'(a) for the backward.
        grouped_gemm(res.recv_x, self.w1.detach().transpose(1, 2), res.expert_offsets, out=h,
                     activation="gelu_save_grad", aux_out=pre, **kw)
        self._mark("fwd_gemm1")
        y = disp.expert_out_buffer(res.handle)
        grouped_gemm(h, self.w2.detach().transpose(1, 2), res.expert_offsets, out=y, **kw)
        self._mark("fwd_gemm2")
        out, ev = disp.combine(y, res.handle, weighted=True, num_sms=self.solo_comm_blocks,
                               inline=True)
        ev.current_stream_wait()
        self._mark("fwd_combine")
        return out, dict(res=res, pre=pre, h=h)

    def _train_backward(self, state: dict, dout: torch.Tensor):
        disp, res = self.dispatcher, state["res"]
        if disp.last_epoch != res.handle.epoch:
            # The forward's receive rows and expert outputs stay in its exchange slot;
            # the backward reads them and its own dispatch takes the other slot, so no
            # dispatch may run in between.
            raise RuntimeError("another dispatch ran on this layer between its forward and backward; "
                               "run backward before the layer's next forward")
        self._mark("bwd_start")
        dout = dout.to(torch.bfloat16).contiguous()
        kw = dict(num_sms=self.gemm_sms, use_atomic_queue=self.use_atomic, work_counter=self.counter)
        # d/d topk weight: <dout[t], y(t, j)>, read from the forward's expert outputs.
        dw = disp.topk_weight_grad(dout, res.handle, num_sms=self.solo_comm_blocks)
        self._mark("bwd_topk_weight_grad")
        # The output gradient goes back to the experts weighted: dY = w * dout rows,
        # laid out exactly like the forward rows: a cached dispatch on the forward's
        # handle (same routing, alignment and receive layout; no layout/count phase).
        rb = disp.dispatch(dout, handle=res.handle, exact_size=False, pad_rows=False, inline=True,
                           scale_rows=True, num_sms=self.solo_comm_blocks)
        rb.event.current_stream_wait()
        self._mark("bwd_dispatch")
        d_pre = torch.empty_like(state["pre"])
        grouped_gemm(rb.recv_x, self.w2.detach(), rb.expert_offsets, out=d_pre, activation="mul_aux",
                     aux_in=state["pre"], **kw)
        self._mark("bwd_dgrad2")
        dx_rows = disp.expert_out_buffer(rb.handle)
        grouped_gemm(d_pre, self.w1.detach(), rb.expert_offsets, out=dx_rows, **kw)
        self._mark("bwd_dgrad1")
        # The combine of dx runs on the exchange stream under the weight gradients.
        dx, ev = disp.combine(dx_rows, rb.handle, weighted=False)
        dw2 = grouped_gemm_wgrad(rb.recv_x, state["h"], rb.expert_offsets, num_sms=self.gemm_sms)
        self._mark("bwd_wgrad2")
        dw1 = grouped_gemm_wgrad(d_pre, res.recv_x, rb.expert_offsets, num_sms=self.gemm_sms)
        self._mark("bwd_wgrad1")
        ev.current_stream_wait()
        self._mark("bwd_combine_tail")
        return dx, dw, dw1, dw2

    def close(self) -> None:
        self.dispatcher.close()


class RoutedExperts(torch.autograd.Function):
    """Autograd node of the routed experts (x, top-k weights, W1, W2 -> out)."""

    @staticmethod
    def forward(ctx, x, topk_w, w1, w2, topk_idx, layer):
        out, state = layer._train_forward(x, topk_idx, topk_w)
        ctx.layer, ctx.state = layer, state
        return out

    @staticmethod
    def backward(ctx, dout):
        dx, dw, dw1, dw2 = ctx.layer._train_backward(ctx.state, dout)
        ctx.state = None
        return dx, dw, dw1, dw2, None, None


def graph_kernel_counts(graph: "torch.cuda.CUDAGraph") -> Optional[dict]:
    """Kernel nodes of a captured graph (made with ``keep_graph=True`` and not yet
    instantiated): ``total``, and ``ours``, those of this library (kernels named in
    namespace ``moe``).  One replay launches exactly these.  None when the driver
    bindings cannot tell (nothing is guessed)."""
    try:
        from cuda.bindings import driver as cu

        ok = cu.CUresult.CUDA_SUCCESS
        g = cu.CUgraph(graph.raw_cuda_graph())
        err, _, n = cu.cuGraphGetNodes(g, 0)
        if err != ok:
            return None
        err, nodes, n = cu.cuGraphGetNodes(g, n)
        if err != ok:
            return None
        total = ours = 0
        for node in nodes[:n]:
            err, kind = cu.cuGraphNodeGetType(node)
            if err != ok:
                return None
            if kind != cu.CUgraphNodeType.CU_GRAPH_NODE_TYPE_KERNEL:
                continue
            total += 1
            err, prm = cu.cuGraphKernelNodeGetParams(node)
            if err != ok or int(prm.func) == 0:
                return None
            err, name = cu.cuFuncGetName(prm.func)
            if err != ok:
                return None
            if bytes(name).startswith(b"_ZN3moe"):
                ours += 1
        return {"total": total, "ours": ours}
    except Exception:  # bindings absent or a different API shape: no count
        return None


class TrainStepGraph:
    """One training step of ``layer`` (forward_autograd + backward) as a CUDA graph.

    ``x`` and ``dout`` are the static inputs: copy each step's data into them
    (under ``torch.no_grad()``) and call ``replay()``.  After a replay ``out``,
    ``probs``, ``topk_idx``, ``x.grad`` and the parameters' ``.grad`` hold that
    step's results (written in place, not accumulated).  The exchange switches to
    device-drawn epochs (DeepEPDispatcher.use_device_epochs) so that every replay
    runs with fresh ones; a step holds two dispatches, which keeps the slot
    alternation aligned across replays.  With a process group, every rank must
    build and replay its graph in step.
    """

    def __init__(self, layer: MoELayer, x: torch.Tensor, dout: torch.Tensor, warmup: int = 2):
        self.layer, self.x, self.dout = layer, x, dout
        disp = layer.dispatcher
        disp.use_device_epochs()
        self.params = [p for p in (layer.router_w, layer.router_b, layer.w1, layer.w2)
                       if p is not None and p.requires_grad]
        cur = torch.cuda.current_stream(layer.device)
        side = torch.cuda.Stream(layer.device)
        side.wait_stream(cur)
        with torch.cuda.stream(side):
            for _ in range(max(1, warmup)):
                self._clear_grads()
                out, _, _ = layer.forward_autograd(x)
                out.backward(dout)
                # Drop the warm-up's autograd graph: a node kept alive from it would keep
                # the parameters' AccumulateGrad nodes bound to this side stream, not to
                # the capture stream that produces the captured step's gradients.
                del out
        cur.wait_stream(side)
        torch.cuda.synchronize(layer.device)
        self._clear_grads()
        e0 = disp.last_epoch
        self.graph = torch.cuda.CUDAGraph(keep_graph=True)
        with torch.cuda.graph(self.graph):
            self.out, self.probs, self.topk_idx = layer.forward_autograd(x)
            self.out.backward(dout)
        if (disp.last_epoch - e0) % 2 != 0:
            raise RuntimeError("a captured training step must hold an even number of dispatches")
        self.kernel_counts = graph_kernel_counts(self.graph)  # kernels per replay
        self.graph.instantiate()

    def _clear_grads(self) -> None:
        for p in self.params:
            p.grad = None
        if self.x.requires_grad:
            self.x.grad = None

    def replay(self) -> None:
        self.graph.replay()


class ForwardGraph:
    """``layer(x, routing=routing)`` captured as one CUDA graph (static inputs).

    Copy each batch into ``x`` (and its routing into the ``routing`` tensors, or
    route inside by passing ``routing=None``) and call ``replay()``; ``out`` then
    holds the result.  Uses device-drawn exchange epochs like TrainStepGraph, and
    needs an even number of chunks per forward (chunk_plan) so that replays keep
    the slot alternation.  With a process group every rank must capture and replay
    in step.
    """

    def __init__(self, layer: MoELayer, x: torch.Tensor, routing=None, warmup: int = 2):
        self.layer, self.x, self.routing = layer, x, routing
        n_chunks = len(layer.chunk_plan(x.shape[0]))
        if n_chunks % 2 != 0:
            raise ValueError(f"a captured forward needs an even number of chunks (has {n_chunks}); "
                             "adjust micro_batch_size")
        layer.dispatcher.use_device_epochs()
        cur = torch.cuda.current_stream(layer.device)
        side = torch.cuda.Stream(layer.device)
        side.wait_stream(cur)
        with torch.cuda.stream(side):
            for _ in range(max(1, warmup)):
                layer(x, routing=routing)
        cur.wait_stream(side)
        torch.cuda.synchronize(layer.device)
        self.graph = torch.cuda.CUDAGraph(keep_graph=True)
        with torch.cuda.graph(self.graph):
            self.out, _ = layer(x, routing=routing)
        self.kernel_counts = graph_kernel_counts(self.graph)  # kernels per replay
        self.graph.instantiate()

    def replay(self) -> None:
        self.graph.replay()
