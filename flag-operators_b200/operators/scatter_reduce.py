"""scatter_reduce — drop-in for operators/scatter_reduce.py of Flag-Operators.

Public API as the reference (scatter_reduce.py:382-468):
    scatter_reduce_(inp, dim, index, src, reduce, *, include_self=True) -> inp
    scatter_reduce(inp, dim, index, src, reduce, *, include_self=True)  -> new tensor
    scatter_reduce_out(out, inp, dim, index, src, reduce, *, include_self=True) -> out
with torch.Tensor.scatter_reduce_ semantics (the reference's CPU branch):
include_self=False keeps self in cells no index reaches, integer mean rounds
toward -inf, amax/amin propagate NaN.  1-4-D tensors, any strides, reduce in
{sum, prod, mean, amax, amin}; dtypes float32/float16/bfloat16/int32/int64.

Kernels: csrc/scatter_reduce.cu (entry point fo_scatter_reduce).  Scratch
(accumulator, counts, and for many 1-D updates the destination-binned pass's
(cell, value) pairs) is allocated here with torch and passed in.
Indices outside [0, self.size(dim)) are skipped on the device and counted;
set FLAGOPS_CHECK_INDEX=1 to make the call synchronise and raise, as torch's
CPU path does.
"""
from __future__ import annotations

import logging
import os

import torch

from . import _lib

logger = logging.getLogger(__name__)

_VALID_REDUCES = frozenset(["sum", "prod", "amax", "amin", "mean"])
_CODE = {"sum": 0, "prod": 1, "mean": 2, "amax": 3, "amin": 4}
_CHECK = os.environ.get("FLAGOPS_CHECK_INDEX", "0") == "1"


def _launch(out: torch.Tensor, dim: int, index: torch.Tensor, src: torch.Tensor, reduce: str,
            include_self: bool) -> None:
    """Scatters src into out (which holds self's values) — the reference's _launch
    (scatter_reduce.py:327-375) without its extra count / clamp / div passes."""
    assert reduce in _VALID_REDUCES, f"Unsupported reduce: {reduce!r}"
    if out.dim() == 0:
        out_v, index_v, src_v = out.view(1), index.view(1), src.view(1)
    else:
        out_v, index_v, src_v = out, index, src
    ndim = out_v.dim()
    assert 1 <= ndim <= 4, f"scatter_reduce supports 1–4-D tensors, got {ndim}D"
    if index_v.dim() != ndim or src_v.dim() != ndim:
        raise RuntimeError("scatter_reduce(): index, self and src must have the same number of "
                           "dimensions")
    if dim < 0:
        dim += ndim
    if not 0 <= dim < ndim:
        raise IndexError(f"scatter_reduce(): dim {dim} out of range")
    if src.dtype != out.dtype:
        raise RuntimeError(f"scatter_reduce(): expected self.dtype to be equal to src.dtype "
                           f"({out.dtype} vs {src.dtype})")
    if index.dtype not in (torch.int64, torch.int32):
        raise RuntimeError("scatter_reduce(): Expected dtype int64 for index")
    for d in range(ndim):
        if index_v.shape[d] > src_v.shape[d] or (d != dim and index_v.shape[d] > out_v.shape[d]):
            raise RuntimeError(f"scatter_reduce(): index size {index_v.shape[d]} exceeds self/src "
                               f"size at dim {d}")
    if not (out.is_cuda and index.is_cuda and src.is_cuda):
        raise RuntimeError("scatter_reduce: self, index and src must all be CUDA tensors")
    if out.numel() == 0:
        return
    code = _CODE[reduce]
    dt = _lib.dtype_code(out.dtype)
    ws_bytes = _lib.ctypes.c_int64(0)
    span = 1 + sum((s - 1) * st for s, st in zip(out_v.shape, out_v.stride()))
    _lib.call("fo_scatter_reduce_workspace_bytes", span, code, int(include_self), dt,
              _lib.ctypes.byref(ws_bytes))
    total = ws_bytes.value
    if ndim == 1 and index_v.stride(0) == 1 and src_v.stride(0) == 1:
        # room for the destination-binned pass (many updates into a bounded output)
        bin_bytes = _lib.ctypes.c_int64(0)
        _lib.call("fo_scatter_reduce_binned_bytes", span, index_v.numel(), code, dt,
                  _lib.ctypes.byref(bin_bytes))
        total += bin_bytes.value
    ws = torch.empty(max(total, 1), dtype=torch.uint8, device=out.device)
    ws_bytes = _lib.ctypes.c_int64(total)
    err = torch.zeros(1, dtype=torch.int32, device=out.device) if _CHECK else None
    _lib.call("fo_scatter_reduce", _lib.ptr(out_v), _lib.ptr(src_v), _lib.ptr(index_v), ndim,
              _lib.i64_array(index_v.shape), _lib.i64_array(index_v.stride()),
              _lib.i64_array(src_v.stride()), _lib.i64_array(out_v.shape),
              _lib.i64_array(out_v.stride()), dim, code, int(bool(include_self)), dt,
              _lib.dtype_code(index.dtype), _lib.ptr(ws), ws_bytes.value, _lib.ptr(err),
              _lib.stream_of(out))
    if err is not None and int(err.item()) != 0:
        raise RuntimeError(f"scatter_reduce(): {int(err.item())} index value(s) out of bounds "
                           f"for dimension {dim} with size {out_v.shape[dim]}")


def scatter_reduce_(
    inp: torch.Tensor,
    dim: int,
    index: torch.Tensor,
    src: torch.Tensor,
    reduce: str,
    *,
    include_self: bool = True,
) -> torch.Tensor:
    """In place: inp.scatter_reduce_(dim, index, src, reduce) (scatter_reduce.py:382-409)."""
    logger.debug("FLAG-OPS SCATTER_REDUCE_ reduce=%s dim=%d", reduce, dim)
    _lib.require_cuda(inp, "scatter_reduce_")
    assert reduce in _VALID_REDUCES, f"Unsupported reduce: {reduce!r}"
    _launch(inp, dim, index, src, reduce, include_self)
    return inp


def scatter_reduce(
    inp: torch.Tensor,
    dim: int,
    index: torch.Tensor,
    src: torch.Tensor,
    reduce: str,
    *,
    include_self: bool = True,
) -> torch.Tensor:
    """Out of place; inp is unchanged (scatter_reduce.py:412-438)."""
    logger.debug("FLAG-OPS SCATTER_REDUCE reduce=%s dim=%d", reduce, dim)
    _lib.require_cuda(inp, "scatter_reduce")
    assert reduce in _VALID_REDUCES, f"Unsupported reduce: {reduce!r}"
    out = inp.clone()
    _launch(out, dim, index, src, reduce, include_self)
    return out


def scatter_reduce_out(
    out: torch.Tensor,
    inp: torch.Tensor,
    dim: int,
    index: torch.Tensor,
    src: torch.Tensor,
    reduce: str,
    *,
    include_self: bool = True,
) -> torch.Tensor:
    """Into an explicit output buffer (scatter_reduce.py:441-468)."""
    logger.debug("FLAG-OPS SCATTER_REDUCE_OUT reduce=%s dim=%d", reduce, dim)
    _lib.require_cuda(inp, "scatter_reduce_out")
    assert reduce in _VALID_REDUCES, f"Unsupported reduce: {reduce!r}"
    if out.shape != inp.shape:
        out.resize_(inp.shape)
    out.copy_(inp)
    _launch(out, dim, index, src, reduce, include_self)
    return out
