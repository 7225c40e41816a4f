"""CPU oracle for the aiter fused-MoE hot path (TEST INFRASTRUCTURE ONLY).

This package restates, in numpy, the reference algorithms of the path that
`aiter_b200` implements on the GPU:

* routing   -- softmax top-k and grouped / biased-grouped top-k
               (op_tests/test_moeTopkSoftmax.py:21-41, aiter/ops/topk.py:116-197)
* sorting   -- moe_sorting_native (op_tests/test_moe_sorting.py:15-70)
* codecs    -- fp8 e4m3fn, bf16, e8m0 and MXFP4 e2m1 number formats
               (aiter/utility/fp4_utils.py:10-107, aiter/ops/quant.py:42-106)
* moe       -- torch_moe_stage1 -> 1x128 requant -> torch_moe_stage2
               (aiter/fused_moe.py:1483-1666, op_tests/test_moe_2stage.py:187-231)
* allreduce -- sum of per-rank partials in fixed rank order

Parity is pinned: `tests/golden/make_golden.py` runs the reference's own torch
functions (loaded from the reference checkout by AST extraction) on seeded inputs
and stores their outputs under `tests/golden/`; `tests/test_oracle_golden.py`
checks every function here against those fixtures.

Only `tests/`, `__graft_entry__.smoke()` and the `cpu_baseline` leg of `bench.py`
may import this package, and only as the checker.  The product path
(`aiter_b200`) never calls into it.
"""
