"""flag-operators_b200: B200 (sm_100a) drop-in for Flag-Operators' operators.* modules.

Submodules mirror the reference package layout (operators/<op>.py):
rms_norm, median, scatter_reduce, fused_cross_entropy, chunk_gated_delta_rule.
Every public function runs hand-written sm_100a kernels through the C ABI in
lib/libflagops.so (declared in include/flagops.h).
"""
