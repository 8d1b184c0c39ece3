"""Drop-in replacement for moe-overlap's ``src/triton_grouped_gemm.py``.

Put ``moe_overlap_b200/shim`` ahead of the reference's ``src`` on ``sys.path``
and ``from triton_grouped_gemm import persistent_grouped_gemm,
reference_grouped_gemm, expert_offsets_from_recv_counts`` (as
``train_moe_baseline.py`` and ``bench_triton_grouped_gemm.py`` do) resolves to
the sm_100a implementation.
"""
import sys
from pathlib import Path

_REPO = Path(__file__).resolve().parents[2]
if str(_REPO) not in sys.path:
    sys.path.insert(0, str(_REPO))

from moe_overlap_b200.gemm import (  # noqa: E402,F401
    expert_offsets_from_recv_counts,
    persistent_grouped_gemm,
    reference_grouped_gemm,
)

__all__ = ["persistent_grouped_gemm", "expert_offsets_from_recv_counts", "reference_grouped_gemm"]
