"""CPU oracle for the MoE expert-GEMM hot path -- TEST INFRASTRUCTURE ONLY.

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline / reference
arm may import anything from this package, and only as the checker or as the
timed CPU baseline.  The product path (moe-gemm-parallel-bench_b200/) never
imports it: there is no CPU fallback.

Parity is pinned: tests/golden/gemm_cases.npz holds outputs of the
reference's own Triton kernels (kernels/grouped_gemm.py:321-482,
kernels/matmul.py:223-273) run here under the Triton CPU interpreter, and
tests/test_oracle.py checks this oracle against them.
"""
