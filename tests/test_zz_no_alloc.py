"""The allocation-free scatter_reduce entry point (fo_scatter_reduce_noalloc).

It exists for callers that cannot allocate device memory when they need a
scatter — a framework that owns the whole device heap, a cgo / JNI / plugin
caller without the program's allocator, code that must avoid the device
synchronisation of cudaMalloc — so its scratch is a static device array inside
the library instead of a caller workspace.  These tests call it through the C
ABI and compare it with fo_scatter_reduce (the entry point that takes a
workspace), within the tolerance of the scatter_reduce parity tests, on two
calls in a row: the second call must not see the first call's scratch.

This file is named to be collected last; it passes alone and after the others.
"""
import ctypes

import pytest
import torch

from operators import _lib

pytestmark = pytest.mark.gpu
DEV = "cuda"
_CODE = {"sum": 0, "prod": 1, "mean": 2, "amax": 3, "amin": 4}


def _args(out, src, index, dim):
    return (_lib.ptr(out), _lib.ptr(src), _lib.ptr(index), out.dim(),
            _lib.i64_array(index.shape), _lib.i64_array(index.stride()),
            _lib.i64_array(src.stride()), _lib.i64_array(out.shape),
            _lib.i64_array(out.stride()), dim)


def _with_workspace(self_, src, index, reduce, include_self, dim=0):
    out = self_.clone()
    code, dt = _CODE[reduce], _lib.dtype_code(out.dtype)
    span = 1 + sum((s - 1) * st for s, st in zip(out.shape, out.stride()))
    nbytes = ctypes.c_int64(0)
    _lib.call("fo_scatter_reduce_workspace_bytes", span, code, int(include_self), dt,
              ctypes.byref(nbytes))
    ws = torch.empty(max(nbytes.value, 1), dtype=torch.uint8, device=DEV)
    _lib.call("fo_scatter_reduce", *_args(out, src, index, dim), code, int(include_self), dt,
              _lib.dtype_code(index.dtype), _lib.ptr(ws), nbytes.value, None,
              _lib.stream_of(out))
    return out


def _no_alloc(self_, src, index, reduce, include_self, dim=0):
    out = self_.clone()
    _lib.call("fo_scatter_reduce_noalloc", *_args(out, src, index, dim), _CODE[reduce],
              int(include_self), _lib.dtype_code(out.dtype), _lib.dtype_code(index.dtype), None,
              _lib.stream_of(out))
    return out


def _no_alloc_view(out, src, index, reduce, include_self, dim=0):
    """In place on `out`, keeping its strides (a view of a larger tensor)."""
    _lib.call("fo_scatter_reduce_noalloc", *_args(out, src, index, dim), _CODE[reduce],
              int(include_self), _lib.dtype_code(out.dtype), _lib.dtype_code(index.dtype), None,
              _lib.stream_of(out))
    return out


def _inputs(seed, n_self=1 << 16, n_src=1 << 20):
    g = torch.Generator().manual_seed(seed)
    self_ = torch.randn(n_self, generator=g)
    src = torch.randn(n_src, generator=g)
    index = torch.randint(0, n_self, (n_src,), generator=g)
    return self_.to(DEV), src.to(DEV), index.to(DEV)


def _close(a, b, reduce, src, index, n_self):
    if reduce in ("amax", "amin"):
        assert torch.equal(a, b)
        return
    # float sums: order-dependent rounding, bounded by 1e-5 * sum(|terms|) per cell
    scale = torch.zeros(n_self, device=DEV, dtype=torch.float64)
    scale.index_add_(0, index, src.abs().double())
    if reduce == "mean":
        cnt = torch.zeros(n_self, device=DEV, dtype=torch.float64)
        cnt.index_add_(0, index, torch.ones_like(src, dtype=torch.float64))
        scale = scale / cnt.clamp(min=1)
    if reduce == "prod":
        torch.testing.assert_close(a, b, rtol=1e-4, atol=1e-30)
        return
    err = (a.double() - b.double()).abs()
    assert bool((err <= 1e-5 * scale + 1e-5).all()), float(err.max())


@pytest.mark.parametrize("reduce,include_self", [("mean", False), ("sum", False),
                                                 ("amax", True), ("prod", False),
                                                 ("mean", True)])
def test_no_alloc_matches_workspace_entry_point_twice(reduce, include_self):
    for seed in (11, 12):   # two calls in a row, different inputs each time
        self_, src, index = _inputs(seed)
        want = _with_workspace(self_, src, index, reduce, include_self)
        got = _no_alloc(self_, src, index, reduce, include_self)
        torch.cuda.synchronize()
        _close(got, want, reduce, src, index, self_.numel())


def test_no_alloc_2d_and_int32():
    g = torch.Generator().manual_seed(3)
    self_ = torch.randint(-50, 50, (64, 300), generator=g, dtype=torch.int32).to(DEV)
    src = torch.randint(-50, 50, (64, 500), generator=g, dtype=torch.int32).to(DEV)
    index = torch.randint(0, 300, (64, 500), generator=g).to(DEV)
    for _ in range(2):
        a = _no_alloc(self_, src, index, "mean", False, dim=1)
        b = _with_workspace(self_, src, index, "mean", False, dim=1)
        assert torch.equal(a, b)


def test_no_alloc_rejects_sizes_beyond_the_static_scratch():
    self_ = torch.zeros(1 << 21, device=DEV)      # 2^21 cells > the 2^20 limit
    src = torch.ones(16, device=DEV)
    index = torch.zeros(16, dtype=torch.int64, device=DEV)
    with pytest.raises(RuntimeError, match="static scratch"):
        _no_alloc(self_, src, index, "mean", False)
    # a reduce that needs no scratch has no limit
    out = _no_alloc(self_, src, index, "sum", True)
    assert out[0].item() == 16.0


def test_no_alloc_limit_is_the_output_memory_span():
    # a column of a [2^19, 4] matrix has 2^19 cells but spans 2^21 - 3 elements
    base = torch.zeros(1 << 19, 4, device=DEV)
    col = base[:, 0]
    src = torch.ones(16, device=DEV)
    index = torch.arange(16, device=DEV)
    with pytest.raises(RuntimeError, match="memory span"):
        _no_alloc_view(col, src, index, "mean", False)
    # the same cells stored contiguously fit
    out = _no_alloc(col.contiguous(), src, index, "mean", False)
    assert out[:16].eq(1.0).all()


def test_no_alloc_argument_errors_match_the_workspace_entry_point():
    src = torch.ones(16, device=DEV)
    index = torch.zeros(16, dtype=torch.int64, device=DEV)
    out = torch.zeros(64, device=DEV)
    bad_shape = _lib.i64_array([-5])
    args = (_lib.ptr(out), _lib.ptr(src), _lib.ptr(index), 1, _lib.i64_array(index.shape),
            _lib.i64_array(index.stride()), _lib.i64_array(src.stride()), bad_shape,
            _lib.i64_array(out.stride()), 0, _CODE["mean"], 0, _lib.dtype_code(out.dtype),
            _lib.dtype_code(index.dtype))
    with pytest.raises(ValueError, match="negative shape") as e1:
        _lib.call("fo_scatter_reduce_noalloc", *args, None, _lib.stream_of(out))
    with pytest.raises(ValueError, match="negative shape") as e2:
        _lib.call("fo_scatter_reduce", *args, None, 0, None, _lib.stream_of(out))
    # same status and message; only the entry point's name in front differs
    assert str(e1.value).split(": ", 1)[1] == str(e2.value).split(": ", 1)[1]
