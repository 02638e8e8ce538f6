"""Argument checks of the C ABI, on a machine without a GPU.

Every entry point validates sizes, pointers, dtypes and options before its
first CUDA call and reports a status code (-1 bad argument -> ValueError, other
codes -> RuntimeError through operators._lib.call) with a message from
fo_last_error().  These calls return before touching a device, so the pointers
below are null or dummy values that are never dereferenced.  Workspace sizes
that are planned on the host (scatter_reduce, the small global median) are
checked against their layout.
"""
import ctypes
import os

import pytest

from operators import _lib

F32, F16, BF16, I32, I64 = 0, 1, 2, 3, 4
SUM, PROD, MEAN, AMAX, AMIN = 0, 1, 2, 3, 4
DUMMY = 0x1000  # a non-null pointer value for checks that only test for null


@pytest.fixture(scope="module", autouse=True)
def _built():
    if not os.path.exists(_lib.LIB_PATH):
        import __graft_entry__
        __graft_entry__.build()


def _arr(vals):
    return (ctypes.c_int64 * len(vals))(*vals)


def _last_error():
    lib = _lib.load()
    lib.fo_last_error.restype = ctypes.c_char_p
    return lib.fo_last_error().decode()


def test_median_dim_sizes():
    with pytest.raises(ValueError, match="negative size"):
        _lib.call("fo_median_dim", None, None, None, -1, 4, F32, None)
    with pytest.raises(ValueError, match="empty dimension"):
        _lib.call("fo_median_dim", None, None, None, 3, 0, F32, None)
    assert "empty dimension" in _last_error()
    _lib.call("fo_median_dim", None, None, None, 0, 0, F32, None)  # no rows: nothing to do
    with pytest.raises(ValueError, match="null pointer"):
        _lib.call("fo_median_dim", None, None, None, 3, 5, F32, None)


def test_median_all_checks_and_small_workspace():
    with pytest.raises(ValueError, match="must not be empty"):
        _lib.call("fo_median_all", DUMMY, DUMMY, 0, F32, None, 0, None)
    with pytest.raises(RuntimeError, match="workspace"):
        _lib.call("fo_median_all", DUMMY, DUMMY, 10, F32, None, 0, None)
    nbytes = ctypes.c_int64(-1)
    _lib.call("fo_median_all_workspace_bytes", 1000, ctypes.byref(nbytes))
    assert nbytes.value == 8  # one CTA below 2^20 elements: the selected index only


def test_rms_norm_sizes():
    _lib.call("fo_rms_norm_fwd", None, None, None, None, 0, 8, 1e-6, F32, F32, None)
    with pytest.raises(ValueError, match="negative size"):
        _lib.call("fo_rms_norm_fwd", None, None, None, None, -2, 8, 1e-6, F32, F32, None)
    with pytest.raises(ValueError, match="must be > 0"):
        _lib.call("fo_rms_norm_fwd", None, None, None, None, 2, 0, 1e-6, F32, F32, None)


def _scatter(ndim=1, dim=0, reduce=SUM, index_dtype=I64, arrays=True):
    one = _arr([4] * 4) if arrays else None
    _lib.call("fo_scatter_reduce", DUMMY, DUMMY, DUMMY, ndim, one, one, one, one, one, dim,
              reduce, 1, F32, index_dtype, None, 0, None, None)


def test_scatter_reduce_argument_checks():
    with pytest.raises(ValueError, match="1-4-D"):
        _scatter(ndim=5)
    with pytest.raises(ValueError, match="dim 3 out of range"):
        _scatter(ndim=2, dim=3)
    with pytest.raises(ValueError, match="Unsupported reduce code 7"):
        _scatter(reduce=7)
    with pytest.raises(ValueError, match="int64 or int32"):
        _scatter(index_dtype=F32)
    with pytest.raises(ValueError, match="null shape"):
        _scatter(arrays=False)


@pytest.mark.parametrize("reduce,include_self,dtype,expect", [
    (SUM, 1, F32, 0),                    # accumulates in out, no scratch
    (SUM, 0, F32, 8 << 20),              # (sum, count) float pairs
    (MEAN, 1, F32, 8 << 20),             # (sum, count) float pairs
    (AMAX, 1, F32, 4 << 20),             # ordered uint32 keys
    (SUM, 1, BF16, 4 << 20),             # fp32 accumulator for 16-bit floats
    (SUM, 1, I32, 0),                    # native int32 atomics in out
    (MEAN, 1, I64, 4 << 20),             # int64 sums in out, int32 counts in scratch
])
def test_scatter_reduce_workspace_plan(reduce, include_self, dtype, expect):
    nbytes = ctypes.c_int64(-1)
    _lib.call("fo_scatter_reduce_workspace_bytes", 1 << 20, reduce, include_self, dtype,
              ctypes.byref(nbytes))
    assert nbytes.value == expect


def test_cross_entropy_argument_checks():
    args = dict(logits=DUMMY, target=DUMMY, loss=DUMMY, lse=DUMMY, out=DUMMY, nvalid=DUMMY)

    def fwd(V=16, ld=16, ls=0.0, reduction=1, dtype=BF16):
        _lib.call("fo_ce_fwd", args["logits"], args["target"], args["loss"], args["lse"],
                  args["out"], args["nvalid"], None, 4, V, ld, -100, ls, reduction, dtype,
                  None, 0, None)

    with pytest.raises(ValueError, match="bad shape"):
        fwd(V=0)
    with pytest.raises(ValueError, match="bad shape"):
        fwd(V=16, ld=8)
    with pytest.raises(RuntimeError, match="unsupported logits dtype"):
        fwd(dtype=I32)
    with pytest.raises(ValueError, match="bad reduction 5"):
        fwd(reduction=5)
    with pytest.raises(ValueError, match="bad label_smoothing"):
        fwd(ls=1.5)


def test_delta_rule_checks():
    with pytest.raises(RuntimeError, match="D=100"):
        _lib.call("fo_gdr_fwd", *([None] * 8), 1, 1, 16, 100, BF16, BF16, None, 0, None)
    with pytest.raises(ValueError, match="negative size"):
        _lib.call("fo_gdr_fwd", *([None] * 8), -1, 1, 16, 128, BF16, BF16, None, 0, None)
    _lib.call("fo_gdr_fwd", *([None] * 8), 0, 4, 16, 128, BF16, BF16, None, 0, None)  # no heads
    with pytest.raises(ValueError, match="N, K in"):
        _lib.call("fo_tc05_selftest", DUMMY, DUMMY, DUMMY, 32, 64, 0, 0, None)


def test_delta_rule_backward_checks():
    bwd_args = lambda B, H, L, D, ws, nbytes: (  # noqa: E731
        *([DUMMY] * 5), None, DUMMY, None, *([DUMMY] * 5), None, B, H, L, D, BF16, BF16, ws,
        nbytes, None)
    with pytest.raises(RuntimeError, match="D=100"):
        _lib.call("fo_gdr_bwd", *bwd_args(1, 1, 16, 100, DUMMY, 1 << 30))
    with pytest.raises(ValueError, match="negative size"):
        _lib.call("fo_gdr_bwd", *bwd_args(-1, 1, 16, 128, DUMMY, 1 << 30))
    _lib.call("fo_gdr_bwd", *bwd_args(0, 4, 16, 128, None, 0))  # no heads: nothing to do
    # workspace: a checkpoint per 16 steps plus one chunk of states, per head
    n = ctypes.c_int64(-1)
    _lib.call("fo_gdr_bwd_workspace_bytes", 2, 3, 70, 64, ctypes.byref(n))
    assert n.value == 6 * (5 + 16) * 64 * 64 * 4
    _lib.call("fo_gdr_bwd_workspace_bytes", 1, 1, 5, 16, ctypes.byref(n))
    assert n.value == (1 + 5) * 16 * 16 * 4
    with pytest.raises(RuntimeError, match="D=48"):
        _lib.call("fo_gdr_bwd_workspace_bytes", 1, 1, 5, 48, ctypes.byref(n))
    need = 6 * (5 + 16) * 64 * 64 * 4
    with pytest.raises(RuntimeError, match="workspace of"):
        _lib.call("fo_gdr_bwd", *bwd_args(2, 3, 70, 64, DUMMY, need - 1))
    with pytest.raises(ValueError, match="16-byte aligned"):
        _lib.call("fo_gdr_bwd", *bwd_args(2, 3, 70, 64, DUMMY + 4, need))
    with pytest.raises(ValueError, match="null pointer"):
        _lib.call("fo_gdr_bwd", *([None] * 14), 1, 1, 8, 16, BF16, BF16, DUMMY, need, None)
