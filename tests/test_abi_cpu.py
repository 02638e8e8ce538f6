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


def test_cpu_tensors_are_rejected_loudly():
    import torch
    from operators.rms_norm import rms_norm
    with pytest.raises(RuntimeError, match="CUDA tensors only"):
        rms_norm(torch.randn(4, 8), (8,), torch.ones(8))
