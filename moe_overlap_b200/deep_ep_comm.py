"""Token dispatch/combine with the call surface of src/deep_ep_comm.py.

``DeepEPDispatcher(group, hidden_size, num_experts, num_sms=24)`` with
``dispatch(x, topk_idx, topk_weights, previous_event=None) -> DispatchResult``
and ``combine(expert_out, handle, previous_event=None) -> (combined_x, event)``
keeps the reference wrapper's names, arguments and results; underneath it is
the NVLink peer-memory exchange of ``libmoe_overlap_b200.so`` (csrc/ep.cu)
instead of DeepEP.

Differences a caller can see, all within the reference's contract:
  * ``recv_x`` has one row per (token, selected local expert), grouped by local
    expert (DeepEP sends one row per (token, rank) in source-rank order).  Each
    row's ``recv_topk_idx``/``recv_topk_weights`` hold the expert in that row's
    slot and -1 / 0 elsewhere, so the reference's per-slot loop
    ``recv_y += experts(recv_x)[slot k] * gate_k`` (src/train_moe_baseline.py:
    394-399) followed by the unweighted ``combine`` gives the same sums.
  * ``DispatchResult`` also carries ``expert_offsets`` (int32 ``[E/W + 1]`` on
    the device) and ``num_recv_tokens_per_expert``: ``recv_x`` can go straight
    into ``persistent_grouped_gemm`` with no sort.
  * With ``exact_size=False`` (DeepEP's ``num_worst_tokens`` mode) nothing
    synchronises with the host: the results are capacity-sized views whose
    unused rows have ``recv_topk_idx == -1``.
  * ``combine(..., weighted=True)`` applies the dispatch's top-k weights inside
    the reduction (fused weighted combine).
  * ``dispatch(x, handle=h)`` is DeepEP's cached mode: new rows on the layout of
    the most recent dispatch ``h``, with no layout or count phase.
  * ``expert_gemm_push`` + ``combine_pushed`` fuse the combine's transfer into the
    down-projection GEMM (its epilogue writes rows to their source ranks);
    ``use_device_epochs`` makes every exchange kernel CUDA-graph-capturable;
    ``inline=True`` runs a phase on the caller's stream.
  * ``num_sms`` counts the exchange kernels' 128-thread blocks, which are sized to
    run beside the persistent GEMM on every SM.
Returned receive tensors are views of the dispatcher's buffers and stay valid
until the dispatch after next (two slots alternate).
"""
from __future__ import annotations

import collections
import os
from dataclasses import dataclass, field
from typing import Optional, Tuple

import torch
import torch.distributed as dist

from . import _lib
from .ep import Endpoint, default_wait_ns


class EventOverlap:
    """CUDA event returned by dispatch/combine (DeepEP's EventOverlap surface)."""

    def __init__(self, event: Optional[torch.cuda.Event] = None):
        self.event = event

    def current_stream_wait(self) -> None:
        if self.event is not None:
            torch.cuda.current_stream().wait_event(self.event)


@dataclass
class DispatchHandle:
    slot: int
    epoch: int
    num_tokens: int
    topk: int
    topk_idx: torch.Tensor
    topk_weights: torch.Tensor
    x: torch.Tensor
    recv_rows: Optional[int]
    combined: bool = False
    stream: Optional[torch.cuda.Stream] = None  # where the dispatch ran, and its end
    event: Optional[torch.cuda.Event] = None
    ordered: bool = False  # expert-ordered: expert_gemm may start before every row landed


@dataclass
class DispatchResult:
    recv_x: torch.Tensor
    recv_topk_idx: torch.Tensor
    recv_topk_weights: torch.Tensor
    handle: object
    event: object
    expert_offsets: Optional[torch.Tensor] = None
    recv_src: Optional[torch.Tensor] = None
    extra: dict = field(default_factory=dict)
    _per_expert: Optional[torch.Tensor] = field(default=None, repr=False)

    @property
    def num_recv_tokens_per_expert(self) -> Optional[torch.Tensor]:
        """Rows per local expert (int32), computed on first access on the caller's
        current stream, after it has waited for the dispatch (no launch otherwise)."""
        if self._per_expert is None and self.expert_offsets is not None:
            ev = getattr(self.event, "event", None)
            if ev is not None:
                torch.cuda.current_stream(self.expert_offsets.device).wait_event(ev)
            offs = self.expert_offsets
            self._per_expert = offs[1:] - offs[:-1]
        return self._per_expert


def exchange_buffers(group, rank: int, world: int, own_base: int, export_handle,
                     import_handle) -> list[int]:
    """Every rank's symmetric buffer as addressable here, indexed by rank.

    Each rank exports an IPC handle for its own buffer, the handles are
    gathered over ``group`` (as DeepEP's Buffer does, buffer.py:96-101), and the
    peers' handles are opened locally; this rank's entry is its own pointer.
    """
    bases = [0] * world
    bases[rank] = own_base
    if world > 1:
        handles = [None] * world
        dist.all_gather_object(handles, export_handle(), group=group)
        for r in range(world):
            if r != rank:
                bases[r] = import_handle(handles[r])
    return bases


def _mark(timeline: list, name: str, stream) -> None:
    ev = torch.cuda.Event(enable_timing=True)
    ev.record(stream)
    timeline.append((name, ev))


def _env_int(name: str, default: int) -> int:
    v = os.environ.get(name)
    return int(v) if v not in (None, "") else default


class DeepEPDispatcher:
    """Intranode dispatch/combine over NVLink peer memory (drop-in for the DeepEP wrapper).

    ``num_sms`` is the grid of the exchange kernels in 128-thread blocks (the
    reference reserves that many SMs for DeepEP, src/train_moe_baseline.py:151-152;
    here the blocks share the SMs with the GEMM instead of taking them from it).
    Capacity: ``max_tokens_per_rank`` tokens per dispatch (env
    ``MOE_B200_MAX_TOKENS``, default 8192), ``max_top_k`` (``MOE_B200_MAX_TOPK``,
    default 8), and ``max_recv_rows`` rows received per rank per dispatch
    (``MOE_B200_MAX_RECV_ROWS``, default world * max_tokens_per_rank *
    min(2, experts per rank)); a dispatch that would exceed it fails on every
    rank with MOE_ERR_CAPACITY instead of writing out of bounds.
    """

    def __init__(self, group: dist.ProcessGroup, hidden_size: int, num_experts: int,
                 num_sms: int = 24, *, max_tokens_per_rank: Optional[int] = None,
                 max_top_k: Optional[int] = None, max_recv_rows: Optional[int] = None,
                 exact_size: bool = True):
        self.group = group
        self.hidden_size = hidden_size
        self.num_experts = num_experts
        self.world = group.size() if group is not None else 1
        self.rank = group.rank() if group is not None else 0
        if num_experts % self.world != 0:
            raise ValueError(f"num_experts ({num_experts}) must be divisible by world_size ({self.world})")
        if hidden_size % 8 != 0:
            raise ValueError("hidden_size must be a multiple of 8 (16-byte rows)")
        self.num_sms = max(1, int(num_sms))
        self.exact_size = exact_size
        self.experts_per_rank = num_experts // self.world
        self.max_tokens = max_tokens_per_rank or _env_int("MOE_B200_MAX_TOKENS", 8192)
        self.max_topk = max_top_k or _env_int("MOE_B200_MAX_TOPK", 8)
        default_rows = self.world * self.max_tokens * min(2, self.experts_per_rank, self.max_topk)
        self.max_recv_rows = max_recv_rows or _env_int("MOE_B200_MAX_RECV_ROWS", default_rows)
        self.device = torch.device("cuda", torch.cuda.current_device())
        self.wait_ns = default_wait_ns()
        self._ep = Endpoint(self.rank, self.world, num_experts, hidden_size, self.max_tokens,
                            self.max_topk, self.max_recv_rows)
        bases = exchange_buffers(group, self.rank, self.world, self._ep.base,
                                 self._ep.export_handle, self._ep.import_handle)
        self._ep.connect(bases)
        if self.world > 1:
            dist.barrier(group=group)
        self.comm_stream = torch.cuda.Stream(self.device)
        self._epoch = 0
        self._device_epochs = False
        self._outstanding: collections.deque[DispatchHandle] = collections.deque()
        self._status = _lib.status_word(self.device)

    # ------------------------------------------------------------------------
    def _enter_comm(self, previous_event, inline: bool = False) -> torch.cuda.Stream:
        """The stream the exchange runs on: the dispatcher's own, after the caller's
        stream and previous_event (the expert outputs handed to combine are produced
        there), or, with ``inline``, the caller's current stream itself."""
        cur = torch.cuda.current_stream(self.device)
        stream = cur if inline else self.comm_stream
        if previous_event is not None:
            ev = getattr(previous_event, "event", previous_event)
            if ev is not None:
                stream.wait_event(ev)
        if not inline:
            self.comm_stream.wait_stream(cur)
        return stream

    def _require_on_device(self, **tensors) -> None:
        """The exchange kernels take raw pointers: every operand must be on this
        dispatcher's GPU (a host pointer handed to a kernel would fault it)."""
        for name, t in tensors.items():
            if t is not None and t.device != self.device:
                raise ValueError(f"{name} must be on {self.device}, not {t.device}")

    def get_dispatch_layout(self, topk_idx: torch.Tensor, num_experts: int):
        """(num_tokens_per_rank, None, num_tokens_per_expert, is_token_in_rank) as DeepEP returns."""
        self._require_on_device(topk_idx=topk_idx)
        idx = topk_idx.to(torch.int64).contiguous()
        t, k = idx.shape
        per_rank = torch.empty(self.world, dtype=torch.int32, device=idx.device)
        per_expert = torch.empty(num_experts, dtype=torch.int32, device=idx.device)
        in_rank = torch.empty(t, self.world, dtype=torch.bool, device=idx.device)
        _lib.check_call(
            _lib.load().moe_ep_dispatch_layout(idx.data_ptr(), t, k, num_experts, self.world,
                                               per_rank.data_ptr(), per_expert.data_ptr(),
                                               in_rank.data_ptr(), _lib.stream_handle(idx.device)),
            "moe_ep_dispatch_layout")
        return per_rank, None, per_expert, in_rank

    def dispatch(self, x: torch.Tensor, topk_idx: Optional[torch.Tensor] = None,
                 topk_weights: Optional[torch.Tensor] = None,
                 previous_event: Optional[object] = None, *,
                 handle: Optional["DispatchHandle"] = None,
                 exact_size: Optional[bool] = None, expert_alignment: int = 1,
                 scale_rows: bool = False, num_sms: Optional[int] = None,
                 pad_rows: Optional[bool] = None, inline: bool = False,
                 timeline: Optional[list] = None, ordered: bool = False) -> DispatchResult:
        """Sends each token's row to the ranks owning its top-k experts.

        With ``ordered`` the tokens travel sorted by the earliest of their experts
        (local expert index first, then owner), so experts complete in that order,
        and each owner counts, per local expert, the rows that have landed; ``extra["scatter_event"]`` of
        the result marks the end of this rank's sending, and ``expert_gemm`` enqueued
        behind it starts each expert's tiles as soon as that expert's rows are all
        here (``event`` still marks every row landed).  Same rows, layout and
        metadata as the default; bf16 rows without ``expert_alignment``/``scale_rows``.

        ``timeline`` (a list) receives (phase, CUDA event) pairs recorded on the
        exchange stream: ``start``, then one after each of the dispatch's three
        launches: ``layout_count`` (per-expert ranks and the count push),
        ``scatter`` (rows pushed to their owners) and ``wait`` (every peer's rows
        landed here).

        With ``handle`` (the handle of the most recent dispatch; ``topk_idx`` and
        ``topk_weights`` then stay None, as in DeepEP's cached mode,
        deep_ep/buffer.py:383-390) the rows of ``x`` go to the places that dispatch
        gave its tokens: no layout or count phase, the same receive layout,
        expert offsets and metadata, and with ``scale_rows`` that dispatch's
        weights.  The result carries a new handle for the combine.
        """
        if isinstance(x, (tuple, list)) or x.dtype != torch.bfloat16:
            # the reference wrapper's bf16-only contract; FP8 goes through dispatch_fp8
            raise RuntimeError("This baseline expects BF16 path (tensor), not FP8 tuple.")
        if x.dim() != 2 or x.size(1) != self.hidden_size:
            raise ValueError(f"x must be [num_tokens, {self.hidden_size}]")
        self._require_on_device(x=x, topk_idx=topk_idx, topk_weights=topk_weights)
        if handle is not None:
            if topk_idx is not None or topk_weights is not None:
                raise ValueError("a cached dispatch takes the routing from its handle: "
                                 "pass topk_idx=None and topk_weights=None")
            return self._dispatch_cached(x, handle, previous_event, exact_size, scale_rows,
                                         num_sms, pad_rows, inline)
        if topk_idx is None or topk_weights is None:
            raise ValueError("dispatch needs topk_idx and topk_weights (or the handle of a dispatch)")
        if topk_idx.dim() != 2 or topk_idx.shape[0] != x.shape[0] or topk_weights.shape != topk_idx.shape:
            raise ValueError("topk_idx and topk_weights must be [num_tokens, top_k]")
        num_tokens, topk = topk_idx.shape
        if num_tokens > self.max_tokens or topk > self.max_topk:
            raise ValueError(
                f"dispatch of {num_tokens} tokens x top-{topk} exceeds the dispatcher's capacity "
                f"({self.max_tokens} x {self.max_topk}); raise MOE_B200_MAX_TOKENS / MOE_B200_MAX_TOPK")
        if len(self._outstanding) >= 2:
            raise RuntimeError("at most two dispatches may be outstanding; combine the oldest first")
        if not 1 <= int(expert_alignment) <= 4096:
            raise ValueError("expert_alignment must be in [1, 4096]")
        if ordered and (int(expert_alignment) != 1 or scale_rows):
            raise ValueError("an ordered dispatch takes neither expert_alignment nor scale_rows")
        if num_sms is not None and int(num_sms) < 1:
            raise ValueError("num_sms must be at least 1")
        exact = self.exact_size if exact_size is None else exact_size
        if exact and self._device_epochs:
            raise ValueError("exact_size needs host epochs; with device epochs use expert_offsets")
        _lib.check_status(self.device)
        self._epoch += 1
        epoch, slot = self._epoch, self._epoch % 2
        stream = self._enter_comm(previous_event, inline)
        with torch.cuda.stream(stream):
            xc = x.contiguous()
            ic = topk_idx.to(torch.int64).contiguous()
            wc = topk_weights.to(torch.float32).contiguous()
            if xc.data_ptr() % 16 != 0:
                xc = xc.clone()
            # Without an exact size the receive views span the whole slot; pad_rows
            # marks the rows past the received count (-1 ids, zero weights) so the
            # views read like DeepEP's.  Callers that use expert_offsets can skip it.
            pad = (not exact) if pad_rows is None else bool(pad_rows)
            kepoch, blocks = 0 if self._device_epochs else epoch, num_sms or self.num_sms
            scatter_event = None
            if ordered:
                if timeline is not None:
                    _mark(timeline, "start", stream)
                self._ep.dispatch_ordered_begin(xc, ic, wc, slot, kepoch, self._status)
                if timeline is not None:
                    _mark(timeline, "layout_count", stream)
                self._ep.dispatch_ordered_scatter(xc, ic, wc, slot, kepoch, blocks, pad, self.wait_ns,
                                                  self._status)
                scatter_event = torch.cuda.Event()
                scatter_event.record(stream)
                if timeline is not None:
                    _mark(timeline, "scatter", stream)
                self._ep.dispatch_end(slot, kepoch, self.wait_ns, self._status)
                if timeline is not None:
                    _mark(timeline, "wait", stream)
            elif timeline is None:
                self._ep.dispatch(xc, ic, wc, slot, kepoch, blocks, pad, self.wait_ns,
                                  self._status, expert_alignment, scale_rows)
            else:  # the same three launches, with an event before and after each
                _mark(timeline, "start", stream)
                self._ep.dispatch_begin(xc, ic, wc, slot, kepoch, self._status)
                _mark(timeline, "layout_count", stream)
                self._ep.dispatch_scatter(xc, ic, wc, slot, kepoch, blocks, pad, self.wait_ns,
                                          self._status, expert_alignment, scale_rows)
                _mark(timeline, "scatter", stream)
                self._ep.dispatch_end(slot, kepoch, self.wait_ns, self._status)
                _mark(timeline, "wait", stream)
            offs = self._ep.slots[slot].expert_offsets
            event = torch.cuda.Event()
            event.record(stream)
        if not inline and not torch.cuda.is_current_stream_capturing():
            for t in (x, topk_idx, topk_weights):
                t.record_stream(self.comm_stream)
        views = self._ep.slots[slot]
        rows = self._ep.received_rows(slot, epoch) if exact else views.recv_x.shape[0]
        handle = DispatchHandle(slot, epoch, num_tokens, topk, ic, wc, xc, rows if exact else None,
                                stream=stream, event=event, ordered=ordered)
        self._outstanding.append(handle)
        kcols = views.recv_topk_idx.stride(0)
        return DispatchResult(
            recv_x=views.recv_x[:rows],
            recv_topk_idx=views.recv_topk_idx.as_strided((rows, topk), (kcols, 1)),
            recv_topk_weights=views.recv_topk_weights.as_strided((rows, topk), (kcols, 1)),
            handle=handle,
            event=EventOverlap(event),
            expert_offsets=offs,
            recv_src=views.recv_src[:rows],
            extra={"scatter_event": EventOverlap(scatter_event)} if ordered else {},
        )

    def expert_gemm(self, handle: DispatchHandle, weight: torch.Tensor, out: torch.Tensor, *,
                    activation: Optional[str] = None, num_sms: Optional[int] = None,
                    use_atomic_queue: bool = True,
                    work_counter: Optional[torch.Tensor] = None) -> torch.Tensor:
        """``out = act(recv_x @ weight[e])`` over an ordered dispatch's receive rows, on
        the caller's stream, each expert's tiles starting once its rows have landed.

        Enqueue it behind the dispatch's ``extra["scatter_event"]`` (this rank's own
        rows and expected counts are then in place); the kernel itself waits for
        the peers' rows, expert by expert.  ``weight`` is ``[E_local, hidden, N]``
        (strided views such as ``w1.transpose(1, 2)`` accepted) and ``out`` has one
        row per receive row (``[max_recv_rows, N]``); ``activation`` None or "gelu".
        """
        if not isinstance(handle, DispatchHandle) or not handle.ordered:
            raise RuntimeError("expert_gemm needs the handle of an ordered dispatch")
        self._check_slot_live(handle)
        self._require_on_device(weight=weight, out=out, work_counter=work_counter)
        if weight.dtype != torch.bfloat16 or out.dtype != torch.bfloat16:
            raise ValueError("expert_gemm expects bf16 weights and output")
        if weight.dim() != 3 or weight.shape[0] != self.experts_per_rank or \
                weight.shape[1] != self.hidden_size:
            raise ValueError(f"weight must be [{self.experts_per_rank}, {self.hidden_size}, N]")
        n = weight.shape[2]
        if out.dim() != 2 or out.shape[1] != n or out.shape[0] < self.max_recv_rows or \
                out.stride(1) != 1 or out.stride(0) % 8 != 0 or out.data_ptr() % 16 != 0:
            raise ValueError(f"out must be a bf16 [>= {self.max_recv_rows}, {n}] tensor with "
                             "16-byte aligned rows")
        _lib.check_status(self.device)
        if use_atomic_queue and work_counter is None:
            work_counter = torch.zeros(1, dtype=torch.int32, device=self.device)
        sms = num_sms or torch.cuda.get_device_properties(self.device).multi_processor_count
        self._ep.expert_gemm(handle.slot, weight, out, activation, sms, use_atomic_queue,
                             work_counter, self.wait_ns, self._status)
        return out

    def dispatch_fp8(self, x: Tuple[torch.Tensor, torch.Tensor], topk_idx: torch.Tensor,
                     topk_weights: torch.Tensor, previous_event: Optional[object] = None, *,
                     exact_size: Optional[bool] = None, num_sms: Optional[int] = None,
                     pad_rows: Optional[bool] = None, inline: bool = False) -> DispatchResult:
        """Dispatch with an FP8 payload, as DeepEP's ``Buffer.dispatch`` takes one.

        ``x`` is the pair (x_fp8 ``[T, H]`` float8_e4m3fn, x_scales ``[T, H/128]``
        float32) of ``fp8.quantize_fp8`` (thirdParty/DeepEP/deep_ep/buffer.py:338-342);
        both are moved unchanged, so each row crosses NVLink in H + H/32 bytes
        instead of 2H.  ``recv_x`` of the result is the pair (recv_fp8 ``[n, H]``,
        recv_scales ``[n, H/128]``), views of the receive slot in the same
        expert-ordered layout, metadata and offsets as ``dispatch``;
        ``fp8.dequantize_fp8`` rebuilds bf16 rows from them.  The reference's
        wrapper (src/deep_ep_comm.py:97-98) takes bf16 only, so ``dispatch`` keeps
        refusing a tuple and the FP8 form has its own name.
        """
        if not isinstance(x, (tuple, list)) or len(x) != 2:
            raise ValueError("dispatch_fp8 takes x as the pair (x_fp8, x_scales)")
        x8, sc = x
        if x8.dtype != torch.float8_e4m3fn or x8.dim() != 2 or x8.size(1) != self.hidden_size:
            raise ValueError(f"x_fp8 must be float8_e4m3fn [num_tokens, {self.hidden_size}]")
        if self.hidden_size % 128 != 0:
            raise ValueError("an FP8 payload needs a hidden size that is a multiple of 128")
        if sc.dtype != torch.float32 or sc.shape != (x8.shape[0], self.hidden_size // 128):
            raise ValueError(f"x_scales must be float32 [num_tokens, {self.hidden_size // 128}]")
        self._require_on_device(x_fp8=x8, x_scales=sc, topk_idx=topk_idx, topk_weights=topk_weights)
        if topk_idx.dim() != 2 or topk_idx.shape[0] != x8.shape[0] or topk_weights.shape != topk_idx.shape:
            raise ValueError("topk_idx and topk_weights must be [num_tokens, top_k]")
        num_tokens, topk = topk_idx.shape
        if num_tokens > self.max_tokens or topk > self.max_topk:
            raise ValueError(
                f"dispatch of {num_tokens} tokens x top-{topk} exceeds the dispatcher's capacity "
                f"({self.max_tokens} x {self.max_topk}); raise MOE_B200_MAX_TOKENS / MOE_B200_MAX_TOPK")
        if len(self._outstanding) >= 2:
            raise RuntimeError("at most two dispatches may be outstanding; combine the oldest first")
        if num_sms is not None and int(num_sms) < 1:
            raise ValueError("num_sms must be at least 1")
        exact = self.exact_size if exact_size is None else exact_size
        if exact and self._device_epochs:
            raise ValueError("exact_size needs host epochs; with device epochs use expert_offsets")
        _lib.check_status(self.device)
        self._epoch += 1
        epoch, slot = self._epoch, self._epoch % 2
        stream = self._enter_comm(previous_event, inline)
        with torch.cuda.stream(stream):
            xc = x8.contiguous()
            if xc.data_ptr() % 16 != 0:
                xc = xc.clone()
            scc = sc.contiguous()
            ic = topk_idx.to(torch.int64).contiguous()
            wc = topk_weights.to(torch.float32).contiguous()
            pad = (not exact) if pad_rows is None else bool(pad_rows)
            self._ep.dispatch_fp8(xc, scc, ic, wc, slot, 0 if self._device_epochs else epoch,
                                  num_sms or self.num_sms, pad, self.wait_ns, self._status)
            offs = self._ep.slots[slot].expert_offsets
            event = torch.cuda.Event()
            event.record(stream)
        if not inline and not torch.cuda.is_current_stream_capturing():
            for t in (x8, sc, topk_idx, topk_weights):
                t.record_stream(self.comm_stream)
        views = self._ep.slots[slot]
        rows = self._ep.received_rows(slot, epoch) if exact else views.recv_x.shape[0]
        handle = DispatchHandle(slot, epoch, num_tokens, topk, ic, wc, xc, rows if exact else None,
                                stream=stream, event=event)
        self._outstanding.append(handle)
        kcols = views.recv_topk_idx.stride(0)
        return DispatchResult(
            recv_x=(views.recv_fp8[:rows], views.recv_scales[:rows]),
            recv_topk_idx=views.recv_topk_idx.as_strided((rows, topk), (kcols, 1)),
            recv_topk_weights=views.recv_topk_weights.as_strided((rows, topk), (kcols, 1)),
            handle=handle,
            event=EventOverlap(event),
            expert_offsets=offs,
            recv_src=views.recv_src[:rows],
        )

    def _dispatch_cached(self, x, handle, previous_event, exact_size, scale_rows, num_sms, pad_rows,
                         inline) -> DispatchResult:
        if not isinstance(handle, DispatchHandle) or handle.epoch != self._epoch:
            raise RuntimeError("a cached dispatch needs the handle of this dispatcher's most recent dispatch")
        if x.shape[0] != handle.num_tokens:
            raise ValueError(f"x must have the {handle.num_tokens} tokens of the handle's dispatch")
        if len(self._outstanding) >= 2:
            raise RuntimeError("at most two dispatches may be outstanding; combine the oldest first")
        if num_sms is not None and int(num_sms) < 1:
            raise ValueError("num_sms must be at least 1")
        exact = self.exact_size if exact_size is None else exact_size
        if exact and self._device_epochs:
            raise ValueError("exact_size needs host epochs; with device epochs use expert_offsets")
        _lib.check_status(self.device)
        self._epoch += 1
        epoch, slot = self._epoch, self._epoch % 2
        stream = self._enter_comm(previous_event, inline)
        if handle.stream is not None and handle.stream != stream and handle.event is not None:
            # The scatter reads the positions the handle's dispatch wrote on its stream.
            stream.wait_event(handle.event)
        with torch.cuda.stream(stream):
            xc = x.contiguous()
            if xc.data_ptr() % 16 != 0:
                xc = xc.clone()
            pad = (not exact) if pad_rows is None else bool(pad_rows)
            self._ep.dispatch_cached(xc, handle.topk_idx, handle.topk_weights, handle.slot, slot,
                                     0 if self._device_epochs else epoch, num_sms or self.num_sms, pad,
                                     self.wait_ns, self._status, scale_rows)
            offs = self._ep.slots[slot].expert_offsets
            event = torch.cuda.Event()
            event.record(stream)
        if not inline and not torch.cuda.is_current_stream_capturing():
            x.record_stream(self.comm_stream)
        views = self._ep.slots[slot]
        if exact:
            rows = handle.recv_rows if handle.recv_rows is not None else self._ep.received_rows(slot, epoch)
        else:
            rows = views.recv_x.shape[0]
        new = DispatchHandle(slot, epoch, handle.num_tokens, handle.topk, handle.topk_idx,
                             handle.topk_weights, xc, rows if exact else None,
                             stream=stream, event=event)
        self._outstanding.append(new)
        kcols = views.recv_topk_idx.stride(0)
        return DispatchResult(
            recv_x=views.recv_x[:rows],
            recv_topk_idx=views.recv_topk_idx.as_strided((rows, handle.topk), (kcols, 1)),
            recv_topk_weights=views.recv_topk_weights.as_strided((rows, handle.topk), (kcols, 1)),
            handle=new,
            event=EventOverlap(event),
            expert_offsets=offs,
            recv_src=views.recv_src[:rows],
        )

    def use_device_epochs(self) -> None:
        """Switch the exchange kernels to epochs drawn on the device (graph-capturable).

        Collective in effect: every rank must switch before the same dispatch.  The
        device counter starts at the last host epoch, the host keeps alternating
        slots, and a captured region must hold an even number of dispatches so that
        replays leave the slot parity unchanged (layer.TrainStepGraph checks this).
        Receive sizes then come only from ``expert_offsets`` (``exact_size`` is not
        available: the host cannot know a replayed dispatch's epoch).
        """
        if self._device_epochs:
            return
        torch.cuda.synchronize(self.device)
        self._ep.set_device_epoch(self._epoch)
        torch.cuda.synchronize(self.device)
        self._device_epochs = True

    @property
    def device_epochs(self) -> bool:
        return self._device_epochs

    @property
    def last_epoch(self) -> int:
        """Epoch of the most recent dispatch (0 before the first)."""
        return self._epoch

    def _check_slot_live(self, handle: DispatchHandle) -> None:
        if self._epoch - handle.epoch >= 2:
            raise RuntimeError("the dispatch's exchange slot has been reused by a later dispatch")

    def topk_weight_grad(self, grad_out: torch.Tensor, handle: DispatchHandle,
                         num_sms: Optional[int] = None) -> torch.Tensor:
        """d loss / d topk_weights of a combined dispatch: <grad_out[t], y(t, j)> (float32 [T, k]).

        Reads the expert outputs that ``handle``'s combine summed, so call it before
        the dispatch after next reuses that slot.
        """
        self._check_slot_live(handle)
        self._require_on_device(grad_out=grad_out)
        if grad_out.shape != (handle.num_tokens, self.hidden_size):
            raise ValueError(f"grad_out must be [{handle.num_tokens}, {self.hidden_size}]")
        out = torch.empty(handle.num_tokens, handle.topk, dtype=torch.float32, device=self.device)
        g = grad_out.to(torch.bfloat16).contiguous()
        self._ep.topk_weight_grad(g, handle.topk_idx, handle.slot, out, 2 * (num_sms or self.num_sms))
        return out

    def expert_out_buffer(self, handle: DispatchHandle) -> torch.Tensor:
        """The slot's expert-output rows: write here (e.g. as the GEMM's output) to skip a copy."""
        self._check_slot_live(handle)
        return self._ep.slots[handle.slot].expert_out

    def combine(self, expert_out: torch.Tensor, handle: DispatchHandle,
                previous_event: Optional[object] = None, *,
                weighted: bool = False,
                out: Optional[torch.Tensor] = None,
                num_sms: Optional[int] = None, inline: bool = False,
                timeline: Optional[list] = None) -> Tuple[torch.Tensor, object]:
        """Sums, per token, the expert outputs its owners produced for it (in original
        token order); with ``weighted`` each row is scaled by its top-k weight.
        ``timeline`` (a list) receives (phase, CUDA event) pairs recorded on the
        exchange stream: ``start``, ``ready`` (this rank's outputs announced to
        every peer) and ``pull`` (rows pulled and reduced)."""
        if not isinstance(handle, DispatchHandle) or handle.combined:
            raise RuntimeError("combine needs the handle of an outstanding dispatch")
        if expert_out.dtype != torch.bfloat16 or expert_out.dim() != 2 or \
                expert_out.size(1) != self.hidden_size:
            raise ValueError(f"expert_out must be bf16 [rows, {self.hidden_size}]")
        self._require_on_device(expert_out=expert_out, out=out)
        if self._outstanding and self._outstanding[0] is not handle:
            raise RuntimeError("combine the oldest outstanding dispatch first")
        _lib.check_status(self.device)
        views = self._ep.slots[handle.slot]
        stream = self._enter_comm(previous_event, inline)
        if out is None:
            out = torch.empty((handle.num_tokens, self.hidden_size), dtype=torch.bfloat16,
                              device=self.device)
        elif (out.shape != (handle.num_tokens, self.hidden_size) or out.dtype != torch.bfloat16
              or not out.is_contiguous() or out.data_ptr() % 16 != 0):
            raise ValueError("out must be a contiguous, 16-byte aligned bf16 [num_tokens, hidden]")
        with torch.cuda.stream(stream):
            if expert_out.data_ptr() != views.expert_out.data_ptr():
                rows = expert_out.shape[0]
                if rows > views.expert_out.shape[0]:
                    raise ValueError("expert_out has more rows than the receive buffer")
                views.expert_out[:rows].copy_(expert_out)
            kepoch = 0 if self._device_epochs else handle.epoch
            if timeline is None:
                self._ep.combine(handle.topk_idx, handle.topk_weights, handle.slot, kepoch,
                                 weighted, out, num_sms or self.num_sms, self.wait_ns, self._status)
            else:  # the same two launches, with an event before and after each
                _mark(timeline, "start", stream)
                self._ep.combine_begin(handle.slot, kepoch)
                _mark(timeline, "ready", stream)
                self._ep.combine_end(handle.topk_idx, handle.topk_weights, handle.slot, kepoch,
                                     weighted, out, num_sms or self.num_sms, self.wait_ns,
                                     self._status)
                _mark(timeline, "pull", stream)
            event = torch.cuda.Event()
            event.record(stream)
        # (under CUDA-graph capture the graph keeps its memory; nothing to record)
        if not inline and not torch.cuda.is_current_stream_capturing():
            expert_out.record_stream(self.comm_stream)
            out.record_stream(self.comm_stream)
        handle.combined = True
        self._outstanding.popleft()
        return out, EventOverlap(event)

    def expert_gemm_push(self, h: torch.Tensor, weight: torch.Tensor, handle: DispatchHandle, *,
                         num_sms: Optional[int] = None, use_atomic_queue: bool = True,
                         work_counter: Optional[torch.Tensor] = None) -> None:
        """Down-projection fused with the combine's transfer, on the caller's stream.

        ``h`` [rows, K] are the expert hidden rows in ``handle``'s receive layout and
        ``weight`` [E_local, K, hidden] (strided views accepted, e.g. ``w2.transpose(1, 2)``
        of nn.Linear weights).  Each result row is written by the GEMM epilogue straight
        into the combine rows of the token's source rank; finish with
        ``combine_pushed(handle, ...)``.
        """
        self._check_slot_live(handle)
        self._require_on_device(h=h, weight=weight, work_counter=work_counter)
        if h.dtype != torch.bfloat16 or weight.dtype != torch.bfloat16:
            raise ValueError("expert_gemm_push expects bf16 rows and weights")
        if weight.dim() != 3 or weight.shape[0] != self.experts_per_rank or \
                weight.shape[2] != self.hidden_size or weight.shape[1] != h.shape[1]:
            raise ValueError(f"weight must be [{self.experts_per_rank}, {h.shape[1]}, {self.hidden_size}]")
        _lib.check_status(self.device)
        if use_atomic_queue and work_counter is None:
            work_counter = torch.zeros(1, dtype=torch.int32, device=self.device)
        sms = num_sms or torch.cuda.get_device_properties(self.device).multi_processor_count
        hc = h if (h.stride(1) == 1 and h.stride(0) % 8 == 0 and h.data_ptr() % 16 == 0) else h.contiguous()
        self._ep.push_gemm(hc, weight, handle.slot, 0 if self._device_epochs else handle.epoch, sms,
                           use_atomic_queue, work_counter, self._status)

    def combine_pushed(self, handle: DispatchHandle, previous_event: Optional[object] = None, *,
                       weighted: bool = False, out: Optional[torch.Tensor] = None,
                       num_sms: Optional[int] = None, inline: bool = False):
        """combine() for rows pushed by ``expert_gemm_push``: a local reduce after every
        owner's GEMM has landed its rows here.  Returns (combined_x, event)."""
        if not isinstance(handle, DispatchHandle) or handle.combined:
            raise RuntimeError("combine needs the handle of an outstanding dispatch")
        if self._outstanding and self._outstanding[0] is not handle:
            raise RuntimeError("combine the oldest outstanding dispatch first")
        _lib.check_status(self.device)
        stream = self._enter_comm(previous_event, inline)
        if out is None:
            out = torch.empty((handle.num_tokens, self.hidden_size), dtype=torch.bfloat16,
                              device=self.device)
        elif (out.shape != (handle.num_tokens, self.hidden_size) or out.dtype != torch.bfloat16
              or not out.is_contiguous() or out.data_ptr() % 16 != 0):
            raise ValueError("out must be a contiguous, 16-byte aligned bf16 [num_tokens, hidden]")
        with torch.cuda.stream(stream):
            self._ep.combine_pushed(handle.topk_idx, handle.topk_weights, handle.slot,
                                    0 if self._device_epochs else handle.epoch, weighted, out,
                                    num_sms or self.num_sms, self.wait_ns, self._status)
            event = torch.cuda.Event()
            event.record(stream)
        if not inline and not torch.cuda.is_current_stream_capturing():
            out.record_stream(self.comm_stream)
        handle.combined = True
        self._outstanding.popleft()
        return out, EventOverlap(event)

    def close(self) -> None:
        """Collective: every rank unmaps its peers' buffers before any rank frees its own."""
        if self._ep is not None:
            torch.cuda.synchronize(self.device)
            if self.world > 1:
                dist.barrier(group=self.group)
            self._ep.close_imports()
            if self.world > 1:
                dist.barrier(group=self.group)
            self._ep.close()
            self._ep = None
