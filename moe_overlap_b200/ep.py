"""Host side of the expert-parallel token exchange (NVLink peer memory).

``Endpoint`` wraps one rank's ``moe_ep_t`` from the C ABI and exposes its
symmetric buffer as zero-copy torch views.  ``LocalGroup`` connects several
endpoints that live on the same GPU in one process; it runs each phase for
every rank before the next phase starts, so no kernel ever waits for a launch
that comes after it.  It is how the multi-rank exchange is exercised on a
single GPU.  Multi-process use goes through ``DeepEPDispatcher``
(``deep_ep_comm.py``), which shares the buffers with CUDA IPC.
"""
from __future__ import annotations

import ctypes
import os
from dataclasses import dataclass

import torch

from . import _lib


class _DeviceBytes:
    """Minimal __cuda_array_interface__ exporter that keeps ``owner`` alive."""

    def __init__(self, ptr: int, nbytes: int, owner):
        self.__cuda_array_interface__ = {
            "shape": (nbytes,),
            "typestr": "|u1",
            "data": (ptr, False),
            "version": 3,
            "strides": None,
        }
        self._owner = owner


def device_bytes(ptr: int, nbytes: int, device: torch.device, owner) -> torch.Tensor:
    return torch.as_tensor(_DeviceBytes(ptr, nbytes, owner), device=device)


class _Views(ctypes.Structure):
    _fields_ = [
        ("recv_x", ctypes.c_void_p),
        ("expert_out", ctypes.c_void_p),
        ("recv_topk_idx", ctypes.c_void_p),
        ("recv_topk_weights", ctypes.c_void_p),
        ("recv_src", ctypes.c_void_p),
        ("expert_offsets", ctypes.c_void_p),
        ("send_pos", ctypes.c_void_p),
        ("host_info", ctypes.c_void_p),
        ("cap_rows", ctypes.c_int64),
        ("max_topk", ctypes.c_int32),
        ("arrived", ctypes.c_void_p),
        ("expected", ctypes.c_void_p),
    ]


def default_wait_ns() -> int:
    """Bound on every device-side wait of the exchange (MOE_B200_EP_TIMEOUT_S, default 30 s)."""
    return int(float(os.environ.get("MOE_B200_EP_TIMEOUT_S", "30")) * 1e9)


@dataclass
class SlotViews:
    recv_x: torch.Tensor           # [cap, H] bf16
    expert_out: torch.Tensor       # [cap, H] bf16
    recv_topk_idx: torch.Tensor    # [cap, max_topk] int64
    recv_topk_weights: torch.Tensor  # [cap, max_topk] float32
    recv_src: torch.Tensor         # [cap, 2] int32
    expert_offsets: torch.Tensor   # [E_local + 1] int32
    send_pos: torch.Tensor         # [max_tokens * max_topk] int32
    host_info: ctypes.Array        # mapped host {epoch, rows}
    arrived: torch.Tensor | None = None   # [E_local] int32 view: rows landed per local expert
    expected: torch.Tensor | None = None  # [E_local] int32: rows expected per local expert
    # FP8 payload of a moe_ep_dispatch_fp8, in the same bytes as recv_x (H % 128 == 0)
    recv_fp8: torch.Tensor | None = None     # [cap, H] float8_e4m3fn
    recv_scales: torch.Tensor | None = None  # [cap, H/128] float32


class Endpoint:
    """One rank's exchange endpoint (symmetric buffer + scratch), on the current device."""

    def __init__(self, rank: int, world: int, num_experts: int, hidden: int, max_tokens: int,
                 max_topk: int, max_recv_rows: int):
        self.lib = _lib.load()
        self.rank, self.world, self.num_experts, self.hidden = rank, world, num_experts, hidden
        self.experts_per_rank = num_experts // world
        self.max_tokens, self.max_topk, self.cap_rows = max_tokens, max_topk, max_recv_rows
        self.device = torch.device("cuda", torch.cuda.current_device())
        handle = ctypes.c_void_p()
        _lib.check_call(
            self.lib.moe_ep_create(rank, world, num_experts, hidden, max_tokens, max_topk,
                                   max_recv_rows, ctypes.byref(handle)),
            "moe_ep_create",
        )
        self.handle = handle
        base, nbytes = ctypes.c_void_p(), ctypes.c_uint64()
        _lib.check_call(self.lib.moe_ep_buffer(handle, ctypes.byref(base), ctypes.byref(nbytes)),
                        "moe_ep_buffer")
        self.base, self.nbytes = int(base.value), int(nbytes.value)
        self._imported: list[int] = []
        self.slots = [self._slot_views(s) for s in range(2)]

    def _slot_views(self, slot: int) -> SlotViews:
        v = _Views()
        _lib.check_call(self.lib.moe_ep_views(self.handle, slot, ctypes.byref(v)), "moe_ep_views")
        cap, k, h = int(v.cap_rows), int(v.max_topk), self.hidden
        dev = self.device

        def raw(ptr, nbytes):
            return device_bytes(int(ptr), int(nbytes), dev, self)

        fp8_rows = fp8_scales = None
        if h % 128 == 0 and cap > 0:
            area = raw(v.recv_x, cap * h * 2)
            fp8_rows = area[:cap * h].view(torch.float8_e4m3fn).view(cap, h)
            fp8_scales = area[cap * h:cap * h + cap * (h // 128) * 4].view(torch.float32) \
                .view(cap, h // 128)
        return SlotViews(
            arrived=raw(v.arrived, self.experts_per_rank * 4).view(torch.int32),
            expected=raw(v.expected, self.experts_per_rank * 4).view(torch.int32),
            recv_fp8=fp8_rows,
            recv_scales=fp8_scales,
            recv_x=raw(v.recv_x, cap * h * 2).view(torch.bfloat16).view(cap, h),
            expert_out=raw(v.expert_out, cap * h * 2).view(torch.bfloat16).view(cap, h),
            recv_topk_idx=raw(v.recv_topk_idx, cap * k * 8).view(torch.int64).view(cap, k),
            recv_topk_weights=raw(v.recv_topk_weights, cap * k * 4).view(torch.float32).view(cap, k),
            recv_src=raw(v.recv_src, cap * 8).view(torch.int32).view(cap, 2),
            expert_offsets=raw(v.expert_offsets, (self.experts_per_rank + 1) * 4)
            .view(torch.int32),
            send_pos=raw(v.send_pos, max(1, self.max_tokens * self.max_topk) * 4).view(torch.int32),
            host_info=(ctypes.c_int64 * 2).from_address(int(v.host_info)),
        )

    def _on_device(self, *tensors) -> None:
        """Kernels take raw pointers: every tensor operand must be on this endpoint's GPU."""
        for t in tensors:
            if t is not None and t.device != self.device:
                raise ValueError(f"exchange operands must be on {self.device}, not {t.device}")

    # ------------------------------------------------------------ connection --
    def export_handle(self) -> bytes:
        buf = ctypes.create_string_buffer(64)
        _lib.check_call(self.lib.moe_ipc_export(ctypes.c_void_p(self.base), buf), "moe_ipc_export")
        return buf.raw

    def import_handle(self, handle: bytes) -> int:
        ptr = ctypes.c_void_p()
        _lib.check_call(self.lib.moe_ipc_import(handle, ctypes.byref(ptr)), "moe_ipc_import")
        self._imported.append(int(ptr.value))
        return int(ptr.value)

    def connect(self, peer_bases: list[int]) -> None:
        arr = (ctypes.c_void_p * self.world)(*peer_bases)
        _lib.check_call(self.lib.moe_ep_connect(self.handle, arr), "moe_ep_connect")

    def close_imports(self) -> None:
        """Unmaps the peer buffers imported with import_handle."""
        torch.cuda.synchronize(self.device)
        for ptr in self._imported:
            self.lib.moe_ipc_close(ctypes.c_void_p(ptr))
        self._imported.clear()

    def close(self) -> None:
        if self.handle is None:
            return
        self.close_imports()
        self.lib.moe_ep_destroy(self.handle)
        self.handle = None

    # ---------------------------------------------------------------- phases --
    def _stream(self) -> int:
        return torch.cuda.current_stream(self.device).cuda_stream

    def dispatch_begin(self, x, topk_idx, topk_w, slot, epoch, status):
        self._on_device(x, topk_idx, topk_w)
        t, k = topk_idx.shape
        _lib.check_call(
            self.lib.moe_ep_dispatch_begin(self.handle, x.data_ptr(), topk_idx.data_ptr(),
                                           topk_w.data_ptr(), t, k, slot, epoch,
                                           status.data_ptr(), self._stream()),
            "moe_ep_dispatch_begin")

    def dispatch_scatter(self, x, topk_idx, topk_w, slot, epoch, num_blocks, pad_rows, wait_ns,
                         status, expert_alignment: int = 1, scale_rows: bool = False):
        self._on_device(x, topk_idx, topk_w)
        t, k = topk_idx.shape
        _lib.check_call(
            self.lib.moe_ep_dispatch_scatter(self.handle, x.data_ptr(), topk_idx.data_ptr(),
                                             topk_w.data_ptr(), t, k, slot, epoch, num_blocks,
                                             1 if pad_rows else 0, expert_alignment,
                                             1 if scale_rows else 0, wait_ns, status.data_ptr(),
                                             self._stream()),
            "moe_ep_dispatch_scatter")

    def dispatch_end(self, slot, epoch, wait_ns, status):
        _lib.check_call(
            self.lib.moe_ep_dispatch_end(self.handle, slot, epoch, wait_ns, status.data_ptr(),
                                         self._stream()),
            "moe_ep_dispatch_end")

    def dispatch_cached_begin(self, slot, epoch):
        _lib.check_call(self.lib.moe_ep_dispatch_cached_begin(self.handle, slot, epoch, self._stream()),
                        "moe_ep_dispatch_cached_begin")

    def dispatch_cached_scatter(self, x, topk_idx, topk_w, src_slot, slot, epoch, num_blocks,
                                pad_rows, wait_ns, status, scale_rows: bool = False):
        self._on_device(x, topk_idx, topk_w)
        t, k = topk_idx.shape
        _lib.check_call(
            self.lib.moe_ep_dispatch_cached_scatter(self.handle, x.data_ptr(), topk_idx.data_ptr(),
                                                    topk_w.data_ptr(), t, k, src_slot, slot, epoch,
                                                    num_blocks, 1 if pad_rows else 0,
                                                    1 if scale_rows else 0, wait_ns,
                                                    status.data_ptr(), self._stream()),
            "moe_ep_dispatch_cached_scatter")

    def dispatch_cached(self, x, topk_idx, topk_w, src_slot, slot, epoch, num_blocks, pad_rows,
                        wait_ns, status, scale_rows: bool = False):
        """Rows x for the tokens and top-k choices of the dispatch into ``src_slot``,
        in that dispatch's layout, into ``slot`` (see moe_ep_dispatch_cached)."""
        self._on_device(x, topk_idx, topk_w)
        t, k = topk_idx.shape
        _lib.check_call(
            self.lib.moe_ep_dispatch_cached(self.handle, x.data_ptr(), topk_idx.data_ptr(),
                                            topk_w.data_ptr(), t, k, src_slot, slot, epoch,
                                            num_blocks, 1 if pad_rows else 0,
                                            1 if scale_rows else 0, wait_ns, status.data_ptr(),
                                            self._stream()),
            "moe_ep_dispatch_cached")

    def combine_begin(self, slot, epoch):
        _lib.check_call(self.lib.moe_ep_combine_begin(self.handle, slot, epoch, self._stream()),
                        "moe_ep_combine_begin")

    def combine_end(self, topk_idx, topk_w, slot, epoch, weighted, out, num_blocks, wait_ns,
                    status):
        self._on_device(topk_idx, topk_w, out)
        t, k = topk_idx.shape
        _lib.check_call(
            self.lib.moe_ep_combine_end(self.handle, topk_idx.data_ptr(),
                                        topk_w.data_ptr() if topk_w is not None else None, t, k,
                                        slot, epoch, 1 if weighted else 0, out.data_ptr(),
                                        num_blocks, wait_ns, status.data_ptr(), self._stream()),
            "moe_ep_combine_end")

    def dispatch(self, x, topk_idx, topk_w, slot, epoch, num_blocks, pad_rows, wait_ns, status,
                 expert_alignment: int = 1, scale_rows: bool = False):
        self._on_device(x, topk_idx, topk_w)
        t, k = topk_idx.shape
        _lib.check_call(
            self.lib.moe_ep_dispatch(self.handle, x.data_ptr(), topk_idx.data_ptr(),
                                     topk_w.data_ptr(), t, k, slot, epoch, num_blocks,
                                     1 if pad_rows else 0, expert_alignment,
                                     1 if scale_rows else 0, wait_ns, status.data_ptr(),
                                     self._stream()),
            "moe_ep_dispatch")

    def dispatch_ordered_begin(self, x, topk_idx, topk_w, slot, epoch, status):
        """Begin phase of an expert-ordered dispatch (moe_ep_dispatch_ordered_begin)."""
        self._on_device(x, topk_idx, topk_w)
        t, k = topk_idx.shape
        _lib.check_call(
            self.lib.moe_ep_dispatch_ordered_begin(self.handle, x.data_ptr(), topk_idx.data_ptr(),
                                                   topk_w.data_ptr(), t, k, slot, epoch,
                                                   status.data_ptr(), self._stream()),
            "moe_ep_dispatch_ordered_begin")

    def dispatch_ordered_scatter(self, x, topk_idx, topk_w, slot, epoch, num_blocks, pad_rows,
                                 wait_ns, status):
        """Scatter phase of an expert-ordered dispatch (moe_ep_dispatch_ordered_scatter)."""
        self._on_device(x, topk_idx, topk_w)
        t, k = topk_idx.shape
        _lib.check_call(
            self.lib.moe_ep_dispatch_ordered_scatter(self.handle, x.data_ptr(), topk_idx.data_ptr(),
                                                     topk_w.data_ptr(), t, k, slot, epoch,
                                                     num_blocks, 1 if pad_rows else 0, wait_ns,
                                                     status.data_ptr(), self._stream()),
            "moe_ep_dispatch_ordered_scatter")

    def expert_gemm(self, slot, b, out, activation, num_sms, use_atomic, work_counter, wait_ns,
                    status) -> None:
        """GEMM over ``slot``'s receive rows that starts each expert once its rows have
        landed (moe_ep_expert_gemm); ``b`` [E_local, hidden, N], ``out`` [cap, N]."""
        self._on_device(b, out, work_counter)
        act = {None: _lib.MOE_ACT_NONE, "none": _lib.MOE_ACT_NONE, "gelu": _lib.MOE_ACT_GELU}[activation]
        _lib.check_call(
            self.lib.moe_ep_expert_gemm(self.handle, slot, b.data_ptr(), b.stride(0), b.stride(1),
                                        b.stride(2), out.data_ptr(), out.stride(0), out.shape[1], act,
                                        int(num_sms), 1 if use_atomic else 0,
                                        work_counter.data_ptr() if work_counter is not None else None,
                                        wait_ns, status.data_ptr(), self._stream()),
            "moe_ep_expert_gemm")

    def dispatch_fp8(self, x_fp8, x_scales, topk_idx, topk_w, slot, epoch, num_blocks, pad_rows,
                     wait_ns, status):
        """Dispatch of an e4m3 payload with its per-128 scales (moe_ep_dispatch_fp8)."""
        self._on_device(x_fp8, x_scales, topk_idx, topk_w)
        t, k = topk_idx.shape
        _lib.check_call(
            self.lib.moe_ep_dispatch_fp8(self.handle, x_fp8.data_ptr(), x_scales.data_ptr(),
                                         topk_idx.data_ptr(), topk_w.data_ptr(), t, k, slot, epoch,
                                         num_blocks, 1 if pad_rows else 0, wait_ns,
                                         status.data_ptr(), self._stream()),
            "moe_ep_dispatch_fp8")

    def topk_weight_grad(self, grad_out, topk_idx, slot, out, num_blocks):
        self._on_device(grad_out, topk_idx, out)
        t, k = topk_idx.shape
        _lib.check_call(
            self.lib.moe_ep_topk_weight_grad(self.handle, grad_out.data_ptr(), topk_idx.data_ptr(),
                                             t, k, slot, out.data_ptr(), num_blocks,
                                             self._stream()),
            "moe_ep_topk_weight_grad")

    def combine(self, topk_idx, topk_w, slot, epoch, weighted, out, num_blocks, wait_ns, status):
        self._on_device(topk_idx, topk_w, out)
        t, k = topk_idx.shape
        _lib.check_call(
            self.lib.moe_ep_combine(self.handle, topk_idx.data_ptr(),
                                    topk_w.data_ptr() if topk_w is not None else None, t, k, slot,
                                    epoch, 1 if weighted else 0, out.data_ptr(), num_blocks,
                                    wait_ns, status.data_ptr(), self._stream()),
            "moe_ep_combine")

    def push_gemm(self, a, b, slot, epoch, num_sms, use_atomic, work_counter, status) -> None:
        """Fused down-projection + combine push of ``a`` rows (this rank's receive
        layout of ``slot``) by ``b`` [E_local, K, hidden] (any strides that
        moe_grouped_gemm accepts); see moe_ep_push_gemm."""
        self._on_device(a, b, work_counter)
        _lib.check_call(
            self.lib.moe_ep_push_gemm(self.handle, a.data_ptr(), a.stride(0), b.data_ptr(),
                                      b.stride(0), b.stride(1), b.stride(2), a.shape[0], a.shape[1],
                                      _lib.MOE_DTYPE_BF16, int(num_sms), 1 if use_atomic else 0,
                                      work_counter.data_ptr() if work_counter is not None else None,
                                      slot, epoch, status.data_ptr(), self._stream()),
            "moe_ep_push_gemm")

    def combine_pushed(self, topk_idx, topk_w, slot, epoch, weighted, out, num_blocks, wait_ns,
                       status) -> None:
        self._on_device(topk_idx, topk_w, out)
        t, k = topk_idx.shape
        _lib.check_call(
            self.lib.moe_ep_combine_pushed(self.handle, topk_idx.data_ptr(),
                                           topk_w.data_ptr() if topk_w is not None else None, t, k,
                                           slot, epoch, 1 if weighted else 0, out.data_ptr(),
                                           num_blocks, wait_ns, status.data_ptr(), self._stream()),
            "moe_ep_combine_pushed")

    def set_device_epoch(self, epoch: int) -> None:
        """Sets the device epoch counter (on the current stream): kernels called with
        epoch 0 draw epoch + 1, + 2, ... on the device."""
        _lib.check_call(self.lib.moe_ep_set_device_epoch(self.handle, int(epoch), self._stream()),
                        "moe_ep_set_device_epoch")

    def received_rows(self, slot: int, epoch: int, timeout_s: float = 60.0) -> int:
        """Rows received in ``slot`` for ``epoch``, read from mapped host memory.

        Spins on the host until the scatter kernel has published the count, as
        DeepEP's dispatch does for its receive sizes (deep_ep.cpp:630-653).
        """
        import time

        info = self.slots[slot].host_info
        t0 = time.monotonic()
        while info[0] != epoch:
            if time.monotonic() - t0 > timeout_s:
                raise _lib.MoeError(_lib.MOE_ERR_TIMEOUT, "waiting for the dispatch receive count")
            time.sleep(0)
        rows = int(info[1])
        if rows < 0:
            raise _lib.MoeError(_lib.MOE_ERR_CAPACITY, "dispatch receive buffer too small")
        return rows

    def __del__(self):
        try:
            if self.handle is not None and self.lib is not None:
                self.lib.moe_ep_destroy(self.handle)
                self.handle = None
        except Exception:
            pass


class LocalGroup:
    """``world`` endpoints on the current GPU in this process, wired to each other.

    ``dispatch``/``combine`` run one phase for every rank before the next phase,
    so each bounded wait finds its flag already raised by an earlier launch.
    """

    def __init__(self, world: int, num_experts: int, hidden: int, max_tokens: int, max_topk: int,
                 max_recv_rows: int, num_blocks: int = 16):
        self.world, self.num_blocks = world, num_blocks
        self.eps = [Endpoint(r, world, num_experts, hidden, max_tokens, max_topk, max_recv_rows)
                    for r in range(world)]
        bases = [ep.base for ep in self.eps]
        for ep in self.eps:
            ep.connect(bases)
        self.epoch = 0
        self.status = torch.zeros(1, dtype=torch.int32, device=self.eps[0].device)
        self.wait_ns = default_wait_ns()

    def use_device_epochs(self) -> None:
        """Later phases pass epoch 0: every endpoint draws its epochs on the device."""
        for ep in self.eps:
            ep.set_device_epoch(self.epoch)
        self.device_epochs = True

    def _kernel_epoch(self, epoch: int) -> int:
        return 0 if getattr(self, "device_epochs", False) else epoch

    def dispatch(self, xs, idxs, ws, pad_rows: bool = False, expert_alignment: int = 1,
                 scale_rows: bool = False):
        self.epoch += 1
        slot, epoch = self.epoch % 2, self._kernel_epoch(self.epoch)
        for r, ep in enumerate(self.eps):
            ep.dispatch_begin(xs[r], idxs[r], ws[r], slot, epoch, self.status)
        for r, ep in enumerate(self.eps):
            ep.dispatch_scatter(xs[r], idxs[r], ws[r], slot, epoch, self.num_blocks, pad_rows,
                                self.wait_ns, self.status, expert_alignment, scale_rows)
        for ep in self.eps:
            ep.dispatch_end(slot, epoch, self.wait_ns, self.status)
        return slot, epoch

    def dispatch_ordered(self, xs, idxs, ws, pad_rows: bool = False, end: bool = True):
        """Every rank's expert-ordered dispatch (arrival counters for expert_gemm);
        with ``end=False`` the final wait for every peer's rows is left out."""
        self.epoch += 1
        slot, epoch = self.epoch % 2, self._kernel_epoch(self.epoch)
        for r, ep in enumerate(self.eps):
            ep.dispatch_ordered_begin(xs[r], idxs[r], ws[r], slot, epoch, self.status)
        for r, ep in enumerate(self.eps):
            ep.dispatch_ordered_scatter(xs[r], idxs[r], ws[r], slot, epoch, self.num_blocks, pad_rows,
                                        self.wait_ns, self.status)
        if end:
            for ep in self.eps:
                ep.dispatch_end(slot, epoch, self.wait_ns, self.status)
        return slot, epoch

    def dispatch_fp8(self, xqs, scales, idxs, ws, pad_rows: bool = False):
        """Every rank's FP8 dispatch (e4m3 rows xqs[r], per-128 scales scales[r])."""
        self.epoch += 1
        slot, epoch = self.epoch % 2, self._kernel_epoch(self.epoch)
        for r, ep in enumerate(self.eps):
            ep.dispatch_begin(xqs[r], idxs[r], ws[r], slot, epoch, self.status)
        lib = self.eps[0].lib
        for r, ep in enumerate(self.eps):
            t, k = idxs[r].shape
            # the scatter phase alone (the begin phase ran for every rank above)
            _lib.check_call(
                lib.moe_ep_dispatch_fp8_scatter(ep.handle, xqs[r].data_ptr(), scales[r].data_ptr(),
                                                idxs[r].data_ptr(), ws[r].data_ptr(), t, k, slot,
                                                epoch, self.num_blocks, 1 if pad_rows else 0,
                                                self.wait_ns, self.status.data_ptr(),
                                                ep._stream()),
                "moe_ep_dispatch_fp8_scatter")
        for ep in self.eps:
            ep.dispatch_end(slot, epoch, self.wait_ns, self.status)
        return slot, epoch

    def dispatch_cached(self, xs, idxs, ws, src_slot: int, pad_rows: bool = False,
                        scale_rows: bool = False):
        """Cached re-dispatch of rows xs[r] in the layout of the dispatch into
        ``src_slot`` (which must be the most recent one); idxs/ws are its inputs."""
        if (self.epoch + 1) % 2 == src_slot:
            raise ValueError("a cached dispatch follows the most recent dispatch (the other slot)")
        self.epoch += 1
        slot, epoch = self.epoch % 2, self._kernel_epoch(self.epoch)
        for ep in self.eps:
            ep.dispatch_cached_begin(slot, epoch)
        for r, ep in enumerate(self.eps):
            ep.dispatch_cached_scatter(xs[r], idxs[r], ws[r], src_slot, slot, epoch, self.num_blocks,
                                       pad_rows, self.wait_ns, self.status, scale_rows)
        for ep in self.eps:
            ep.dispatch_end(slot, epoch, self.wait_ns, self.status)
        return slot, epoch

    def push_gemm(self, hs, ws_b, slot, epoch, num_sms=148, work_counter=None):
        """Each rank's fused GEMM + push (rank r: rows hs[r] by weights ws_b[r])."""
        epoch = self._kernel_epoch(epoch)
        for r, ep in enumerate(self.eps):
            ep.push_gemm(hs[r], ws_b[r], slot, epoch, num_sms, work_counter is not None,
                         work_counter, self.status)

    def combine_pushed(self, idxs, ws, slot, epoch, weighted, outs):
        epoch = self._kernel_epoch(epoch)
        for r, ep in enumerate(self.eps):
            ep.combine_pushed(idxs[r], ws[r], slot, epoch, weighted, outs[r], self.num_blocks,
                              self.wait_ns, self.status)

    def combine(self, idxs, ws, slot, epoch, weighted, outs):
        epoch = self._kernel_epoch(epoch)
        for ep in self.eps:
            ep.combine_begin(slot, epoch)
        for r, ep in enumerate(self.eps):
            ep.combine_end(idxs[r], ws[r], slot, epoch, weighted, outs[r], self.num_blocks,
                           self.wait_ns, self.status)

    def close(self):
        for ep in self.eps:
            ep.close()
