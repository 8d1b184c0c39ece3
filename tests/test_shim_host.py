"""The drop-in shims (moe_overlap_b200/shim) resolve the reference's module names.

With the shim directory first on sys.path, ``triton_grouped_gemm`` and
``deep_ep_comm`` must give this package's implementations with the reference's
call signatures (src/triton_grouped_gemm.py:300-304,326-338,446;
src/deep_ep_comm.py:26,69-75,107).  When a checkout of the reference is given
(MOE_REFERENCE_SRC=<checkout>/src), its own scripts train_moe_baseline.py and
bench_triton_grouped_gemm.py are imported unchanged behind the shims and must
bind our functions.  Each check runs in a fresh interpreter (clean sys.path and
module cache); nothing is written into the reference tree.
"""
import os
import subprocess
import sys
from pathlib import Path

import pytest

REPO = Path(__file__).resolve().parents[1]
SHIM = REPO / "moe_overlap_b200" / "shim"

CHECK = r"""
import inspect, sys
sys.dont_write_bytecode = True
sys.path[:0] = [p for p in ({shim!r}, {ref!r}) if p]
import triton_grouped_gemm as tg
import deep_ep_comm as dc
import moe_overlap_b200.gemm as g
import moe_overlap_b200.deep_ep_comm as d

assert tg.persistent_grouped_gemm is g.persistent_grouped_gemm
assert tg.expert_offsets_from_recv_counts is g.expert_offsets_from_recv_counts
assert tg.reference_grouped_gemm is g.reference_grouped_gemm
assert dc.DeepEPDispatcher is d.DeepEPDispatcher

def params(f):
    return [(p.name, p.default) for p in inspect.signature(f).parameters.values()
            if p.kind in (p.POSITIONAL_ONLY, p.POSITIONAL_OR_KEYWORD)]

E = inspect.Parameter.empty
assert params(tg.persistent_grouped_gemm) == [
    ("a_cat", E), ("b_expert", E), ("expert_offsets", E), ("num_sms", 24), ("block_m", 128),
    ("block_n", 128), ("block_k", 32), ("use_atomic_queue", True), ("work_counter", None),
    ("num_warps", 8), ("num_stages", 3)], params(tg.persistent_grouped_gemm)
assert [n for n, _ in params(tg.expert_offsets_from_recv_counts)] == [
    "num_recv_tokens_per_expert", "device", "dtype"]
assert [n for n, _ in params(tg.reference_grouped_gemm)] == ["a_cat", "b_expert", "expert_offsets"]
assert params(dc.DeepEPDispatcher.__init__)[:5] == [
    ("self", E), ("group", E), ("hidden_size", E), ("num_experts", E), ("num_sms", 24)]
assert [n for n, _ in params(dc.DeepEPDispatcher.dispatch)][:5] == [
    "self", "x", "topk_idx", "topk_weights", "previous_event"]
assert [n for n, _ in params(dc.DeepEPDispatcher.combine)] == [
    "self", "expert_out", "handle", "previous_event"]
if {ref!r}:
    import bench_triton_grouped_gemm as b
    import train_moe_baseline as t
    assert b.persistent_grouped_gemm is g.persistent_grouped_gemm
    assert b.reference_grouped_gemm is g.reference_grouped_gemm
    assert t.persistent_grouped_gemm is g.persistent_grouped_gemm
    assert t.DeepEPDispatcher is d.DeepEPDispatcher
print("ok")
"""


def _run(ref: str) -> None:
    env = dict(os.environ, PYTHONDONTWRITEBYTECODE="1")
    r = subprocess.run([sys.executable, "-c", CHECK.format(shim=str(SHIM), ref=ref)], cwd=REPO,
                       capture_output=True, text=True, env=env, timeout=300)
    assert r.returncode == 0 and r.stdout.strip().endswith("ok"), r.stdout + r.stderr


def test_shims_resolve_the_reference_names_with_its_signatures():
    _run("")


def test_reference_scripts_import_unchanged_behind_the_shims():
    ref = os.environ.get("MOE_REFERENCE_SRC", "")
    if not ref or not (Path(ref) / "train_moe_baseline.py").exists():
        pytest.skip("set MOE_REFERENCE_SRC to a checkout's src directory")
    _run(ref)
