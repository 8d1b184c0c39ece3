"""Drop-in replacement for moe-overlap's ``src/deep_ep_comm.py``.

With ``moe_overlap_b200/shim`` ahead of the reference's ``src`` on
``sys.path``, ``from deep_ep_comm import DeepEPDispatcher`` (as
``train_moe_baseline.py:14`` and ``verify_deepep_dispatch.py:25`` do) resolves
to the NVLink peer-memory exchange of this package.
"""
import sys
from pathlib import Path

_REPO = Path(__file__).resolve().parents[2]
if str(_REPO) not in sys.path:
    sys.path.insert(0, str(_REPO))

from moe_overlap_b200.deep_ep_comm import (  # noqa: E402,F401
    DeepEPDispatcher,
    DispatchResult,
    EventOverlap,
)

__all__ = ["DeepEPDispatcher", "DispatchResult", "EventOverlap"]
