"""CPU oracle for the moe_overlap_b200 hot path -- TEST INFRASTRUCTURE ONLY.

A plain numpy restatement of the reference's algorithms (Hongyu15/moe-overlap,
``src/triton_grouped_gemm.py``, ``src/train_moe_baseline.py`` and the intranode
semantics of ``thirdParty/DeepEP``), each function citing the reference lines
it follows.  Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s
CPU-baseline / reference arm may import it, and only as the checker or as the
timed CPU baseline; the product package never imports it.

Parity pin: the restatement is checked against golden vectors produced by
running the reference's own Python code in the build container
(``tests/golden/make_golden.py``; fixtures in ``tests/golden/``).
"""
