"""B200-native (sm_100a) MoE expert hot path: persistent grouped GEMM and
NVLink token dispatch/combine, behind the call surface of moe-overlap's
``triton_grouped_gemm`` and ``deep_ep_comm`` modules.

The compute runs in ``libmoe_overlap_b200.so`` (built in-tree by
``python -m moe_overlap_b200.build``) through its C ABI (``include/moe_overlap.h``).
"""
from .gemm import (
    expert_offsets_from_recv_counts,
    grouped_gemm,
    grouped_gemm_wgrad,
    persistent_grouped_gemm,
    reference_grouped_gemm,
    tile_list,
)
from ._lib import MoeError, check_status
from .fp8 import dequantize_fp8, quantize_fp8
from .router import router_topk

__all__ = [
    "persistent_grouped_gemm",
    "grouped_gemm",
    "grouped_gemm_wgrad",
    "expert_offsets_from_recv_counts",
    "reference_grouped_gemm",
    "tile_list",
    "router_topk",
    "quantize_fp8",
    "dequantize_fp8",
    "MoeError",
    "check_status",
]

# The exchange (deep_ep_comm.DeepEPDispatcher, ep.Endpoint/LocalGroup) and the
# layer (layer.MoELayer, TrainStepGraph, ForwardGraph) are imported from their
# modules; they need torch.distributed only when a process group is given.
