"""Parity oracle — TEST INFRASTRUCTURE ONLY.

CPU restatement of the reference (iamsuperfly/Flag-Operators) CPU path for the
five operators.  Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline
/ reference legs may import this package, and only as the checker or as the
timed CPU baseline.  The product (flag-operators_b200/operators) never imports
it: CUDA tensors always run the sm_100a kernels.

Pinning: every function here is checked in tests/test_oracle_cpu.py against the
golden fixtures in tests/golden/, which tests/golden/make_golden.py produced by
importing the reference's own operators.* modules and running their CPU
branches on seeded inputs (plus the known-answer vectors of the reference's own
tests).  Parity is therefore pinned to the reference itself.
"""
from .ops import (  # noqa: F401
    rms_norm_forward,
    rms_norm_backward,
    median,
    median_dim_np,
    scatter_reduce_,
    scatter_reduce,
    scatter_reduce_out,
    scatter_reduce_scale,
    fused_cross_entropy,
    fused_cross_entropy_grad,
    delta_rule_forward,
    delta_rule_grads,
    delta_rule_backward,
    delta_rule_backward_chunked,
    ce_shard_stats,
    ce_shard_combine,
    ce_rows_partial,
    ce_rows_combine,
)
