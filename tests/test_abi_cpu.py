"""The C-ABI library loads on a machine without a GPU and exports every symbol
that include/flagops.h declares (no compute calls here)."""
import ctypes
import os
import re

import pytest

from conftest import REPO

HEADER = os.path.join(REPO, "include", "flagops.h")


def _declared():
    text = open(HEADER).read()
    return sorted(set(re.findall(r"^FO_API\s+(?:const\s+char\s*\*|int)\s+(fo_\w+)\s*\(",
                                 text, flags=re.M)))


def test_header_declares_entry_points():
    names = _declared()
    for must in ("fo_rms_norm_fwd", "fo_median_dim", "fo_scatter_reduce", "fo_ce_fwd",
                 "fo_ce_bwd", "fo_gdr_fwd", "fo_last_error"):
        assert must in names


def test_library_exports_every_declared_symbol():
    from operators import _lib
    if not os.path.exists(_lib.LIB_PATH):
        import __graft_entry__  # noqa: F401  (build() compiles it)
        __graft_entry__.build()
    lib = ctypes.CDLL(_lib.LIB_PATH)
    missing = [n for n in _declared() if not hasattr(lib, n)]
    assert not missing, f"declared in flagops.h but not exported: {missing}"
    lib.fo_abi_version.restype = ctypes.c_int
    assert lib.fo_abi_version() >= 1


def test_python_signatures_cover_header():
    from operators import _lib
    assert set(_declared()) <= set(_lib.declared_symbols())


def _cpu_calls():
    import torch
    from operators.chunk_gated_delta_rule import chunk_gated_delta_rule
    from operators.fused_cross_entropy import cross_entropy_loss, fused_cross_entropy
    from operators.median import median
    from operators.rms_norm import rms_norm, rms_norm_backward, rms_norm_forward, rms_norm_out
    from operators.scatter_reduce import scatter_reduce, scatter_reduce_, scatter_reduce_out
    x = torch.randn(4, 8)
    idx = torch.randint(0, 4, (6,))
    src, s0 = torch.randn(6), torch.randn(4)
    tgt = torch.randint(0, 8, (4,))
    q = torch.randn(1, 1, 8, 16)
    gate = torch.rand(1, 1, 8)
    return {
        "rms_norm": lambda: rms_norm(x, (8,), torch.ones(8)),
        "rms_norm_forward": lambda: rms_norm_forward(x, (8,), torch.ones(8)),
        "rms_norm_out": lambda: rms_norm_out(torch.empty(4, 8), x, (8,), torch.ones(8)),
        "rms_norm_backward": lambda: rms_norm_backward(x, x, torch.ones(4), (8,), torch.ones(8)),
        "median": lambda: median(x),
        "median_dim": lambda: median(x, dim=1),
        "scatter_reduce": lambda: scatter_reduce(s0, 0, idx, src, "sum"),
        "scatter_reduce_": lambda: scatter_reduce_(s0.clone(), 0, idx, src, "sum"),
        "scatter_reduce_out": lambda: scatter_reduce_out(torch.empty(4), s0, 0, idx, src, "sum"),
        "fused_cross_entropy": lambda: fused_cross_entropy(x, tgt),
        "cross_entropy_loss": lambda: cross_entropy_loss(x, tgt),
        "chunk_gated_delta_rule": lambda: chunk_gated_delta_rule(q, q, q, gate, gate),
    }


@pytest.mark.parametrize("op", sorted(["rms_norm", "rms_norm_forward", "rms_norm_out",
                                       "rms_norm_backward", "median", "median_dim",
                                       "scatter_reduce", "scatter_reduce_", "scatter_reduce_out",
                                       "fused_cross_entropy", "cross_entropy_loss",
                                       "chunk_gated_delta_rule"]))
def test_cpu_tensors_are_rejected_loudly(op):
    """The product path has no CPU fallback: CPU tensors raise instead of being
    computed some other way (the reference's CPU branch lives only in oracle/)."""
    with pytest.raises(RuntimeError, match="CUDA tensors only"):
        _cpu_calls()[op]()
