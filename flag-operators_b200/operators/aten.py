"""PyTorch dispatcher registration of the median and scatter_reduce kernels.

The reference has one optional hook, register_with_flaggems()
(operators/median.py:363-372): it hands `median` to FlagGems' private registry
when that package is installed.  This module registers the same kernels with
PyTorch's own dispatcher instead, as FlagGems' use_gems() does for its Triton
kernels:

* custom ops ``flagops::median``, ``flagops::median_dim`` and
  ``flagops::scatter_reduce`` (functional forms, CUDA only), registered when this
  module is imported, each with a fake kernel, so FX / torch.compile tracing
  knows their output shapes and dtypes without running them;
* ``use_flagops()``, a context manager that overrides ``aten::median``,
  ``aten::median.dim``, ``aten::scatter_reduce.two``,
  ``aten::scatter_reduce_.two`` and ``aten::scatter_reduce.two_out`` for CUDA
  tensors.  Inside it, ``torch.median`` and ``Tensor.scatter_reduce(_)`` on CUDA
  tensors run the sm_100a kernels; on leaving it the registration is dropped and
  PyTorch's own kernels serve those ops again.  Nested blocks share the
  outermost block's registration.

The overrides accept what the kernels accept: median of float32 / float16 /
bfloat16 / int32 / int64 (int8 / int16 / uint8 widened), scatter_reduce of
float32 / float16 / bfloat16 / int32 / int64 on 1-4-D tensors.  Anything else
raises the kernels' error, so enter the context around code that stays within
them.
"""
from __future__ import annotations

import contextlib
import threading
import warnings
from typing import Tuple

import torch

from .median import median as _median
from .scatter_reduce import scatter_reduce as _scatter_reduce
from .scatter_reduce import scatter_reduce_ as _scatter_reduce_
from .scatter_reduce import scatter_reduce_out as _scatter_reduce_out

__all__ = ["use_flagops", "OVERRIDDEN"]

# aten overloads replaced inside use_flagops()
OVERRIDDEN = ("median", "median.dim", "scatter_reduce.two", "scatter_reduce_.two",
              "scatter_reduce.two_out")


# ---------------------------------------------------------------------------
# flagops:: custom ops
# ---------------------------------------------------------------------------
@torch.library.custom_op("flagops::median", mutates_args=(), device_types="cuda")
def _op_median(x: torch.Tensor) -> torch.Tensor:
    return _median(x)


@_op_median.register_fake
def _(x):
    if x.numel() == 0:
        raise RuntimeError("median() input must not be empty")
    return x.new_empty(())


@torch.library.custom_op("flagops::median_dim", mutates_args=(), device_types="cuda")
def _op_median_dim(x: torch.Tensor, dim: int, keepdim: bool = False
                   ) -> Tuple[torch.Tensor, torch.Tensor]:
    r = _median(x, dim, keepdim)
    return r.values, r.indices


def _median_dim_shape(x: torch.Tensor, dim: int, keepdim: bool):
    nd = max(x.dim(), 1)
    d = dim + nd if dim < 0 else dim
    if not 0 <= d < nd:
        raise IndexError(f"median: dim {dim} out of range for a {x.dim()}-D tensor")
    if x.dim() == 0:
        return ()
    shape = list(x.shape)
    if keepdim:
        shape[d] = 1
    else:
        del shape[d]
    return tuple(shape)


@_op_median_dim.register_fake
def _(x, dim, keepdim=False):
    shape = _median_dim_shape(x, dim, keepdim)
    return x.new_empty(shape), x.new_empty(shape, dtype=torch.int64)


@torch.library.custom_op("flagops::scatter_reduce", mutates_args=(), device_types="cuda")
def _op_scatter_reduce(x: torch.Tensor, dim: int, index: torch.Tensor, src: torch.Tensor,
                       reduce: str, include_self: bool = True) -> torch.Tensor:
    return _scatter_reduce(x, dim, index, src, reduce, include_self=include_self)


@_op_scatter_reduce.register_fake
def _(x, dim, index, src, reduce, include_self=True):
    return torch.empty_like(x)


# ---------------------------------------------------------------------------
# aten overrides
# ---------------------------------------------------------------------------
def _aten_median(self):
    return _median(self)


def _aten_median_dim(self, dim, keepdim=False):
    r = _median(self, dim, keepdim)
    return r.values, r.indices


def _aten_scatter_reduce(self, dim, index, src, reduce, *, include_self=True):
    return _scatter_reduce(self, dim, index, src, reduce, include_self=include_self)


def _aten_scatter_reduce_(self, dim, index, src, reduce, *, include_self=True):
    return _scatter_reduce_(self, dim, index, src, reduce, include_self=include_self)


def _aten_scatter_reduce_out(self, dim, index, src, reduce, *, include_self=True, out):
    return _scatter_reduce_out(out, self, dim, index, src, reduce, include_self=include_self)


_IMPLS = {
    "median": _aten_median,
    "median.dim": _aten_median_dim,
    "scatter_reduce.two": _aten_scatter_reduce,
    "scatter_reduce_.two": _aten_scatter_reduce_,
    "scatter_reduce.two_out": _aten_scatter_reduce_out,
}


_lock = threading.Lock()
_depth = 0
_lib_handle = None


@contextlib.contextmanager
def use_flagops():
    """Routes aten median / scatter_reduce on CUDA tensors to the sm_100a kernels
    for the duration of the block.  Re-entrant: nested blocks share the outermost
    block's registration, which is dropped when that block exits."""
    global _depth, _lib_handle
    with _lock:
        if _depth == 0:
            lib = torch.library.Library("aten", "IMPL")
            try:
                with warnings.catch_warnings():
                    # PyTorch warns once that an existing CUDA kernel is overridden
                    warnings.filterwarnings("ignore", message=".*[Oo]verrid.*")
                    for name in OVERRIDDEN:
                        lib.impl(name, _IMPLS[name], "CUDA")
            except BaseException:
                lib._destroy()
                raise
            _lib_handle = lib
        _depth += 1
    try:
        yield
    finally:
        with _lock:
            _depth -= 1
            if _depth == 0:
                _lib_handle._destroy()
                _lib_handle = None
