"""median — drop-in for operators/median.py of Flag-Operators.

median(inp, dim=None, keepdim=False) with torch.median semantics (the reference's
CPU branch, median.py:348-352): lower median; along a dim it returns
torch.return_types.median(values, indices) where the index is the k-th entry of
a stable sort (bit-exact with torch CPU, ties included), -0.0 == +0.0, and a
row with a NaN yields NaN at the index of its first NaN.

Kernels (csrc/median.cu): radix select over an order-preserving key, one warp
per row (row in registers) for rows up to 2048 elements, one CTA per row above.
Supported dtypes: float32, float16, bfloat16, int32, int64 (int8/int16/uint8 are
widened to int32, which preserves order and values).
"""
from __future__ import annotations

import logging

import torch

from . import _lib

logger = logging.getLogger(__name__)

_WIDEN = {torch.int8: torch.int32, torch.int16: torch.int32, torch.uint8: torch.int32}


def _prep(inp: torch.Tensor) -> torch.Tensor:
    if inp.dtype in _WIDEN:
        return inp.to(_WIDEN[inp.dtype])
    _lib.dtype_code(inp.dtype)  # raises for unsupported dtypes
    if inp.dtype == torch.float64:
        raise TypeError("median: float64 is not supported by flag-operators_b200")
    return inp


def _median_dim(inp: torch.Tensor, dim: int, keepdim: bool):
    """Median along `dim` (median.py:241-305): returns (values, indices)."""
    ndim = inp.dim()
    if ndim == 0:
        inp = inp.reshape(1)
        ndim = 1
        squeeze_all = True
    else:
        squeeze_all = False
    if dim < 0:
        dim = ndim + dim
    if not 0 <= dim < ndim:
        raise IndexError(f"median: dim {dim} out of range for a {ndim}-D tensor")
    orig_dtype = inp.dtype
    x = _prep(inp)
    if dim != ndim - 1:
        x = x.movedim(dim, -1)
    x = x.contiguous()
    moved_shape = x.shape
    N = moved_shape[-1]
    M = x.numel() // N if N > 0 else 0
    if N == 0:
        raise IndexError("median(): cannot compute the median of a dimension of size 0")
    vals = torch.empty(M, dtype=x.dtype, device=x.device)
    idx = torch.empty(M, dtype=torch.int64, device=x.device)
    if M > 0:
        _lib.call("fo_median_dim", _lib.ptr(x), _lib.ptr(vals), _lib.ptr(idx), M, N,
                  _lib.dtype_code(x.dtype), _lib.stream_of(x))
    out_shape = list(moved_shape[:-1])
    if keepdim:
        out_shape.append(1)
    vals = vals.reshape(out_shape).to(orig_dtype)
    idx = idx.reshape(out_shape)
    if keepdim and dim != ndim - 1:
        vals = vals.movedim(-1, dim)
        idx = idx.movedim(-1, dim)
    if squeeze_all:
        vals, idx = vals.reshape(()), idx.reshape(())
    return torch.return_types.median([vals, idx])


def _median_global(inp: torch.Tensor) -> torch.Tensor:
    """Median of all elements (median.py:308-325), as a 0-d tensor of inp's dtype."""
    if inp.numel() == 0:
        raise RuntimeError("median() input must not be empty")
    orig_dtype = inp.dtype
    x = _prep(inp).reshape(-1).contiguous()
    out = torch.empty((), dtype=x.dtype, device=x.device)
    nbytes = _lib.ctypes.c_int64(0)
    _lib.call("fo_median_all_workspace_bytes", x.numel(), _lib.ctypes.byref(nbytes))
    ws = torch.empty((nbytes.value + 7) // 8, dtype=torch.int64, device=x.device)
    _lib.call("fo_median_all", _lib.ptr(x), _lib.ptr(out), x.numel(), _lib.dtype_code(x.dtype),
              _lib.ptr(ws), nbytes.value, _lib.stream_of(x))
    return out.to(orig_dtype)


def median(inp: torch.Tensor, dim=None, keepdim: bool = False):
    """torch.median-compatible median (median.py:332-356)."""
    logger.debug("FLAG-OPS MEDIAN dim=%s keepdim=%s", dim, keepdim)
    _lib.require_cuda(inp, "median")
    if dim is None:
        return _median_global(inp)
    return _median_dim(inp, dim, keepdim)


def timeouts() -> int:
    """Hand-off waits of the producer/consumer kernel that ran out of polls since
    load (0 in a healthy run)."""
    c = _lib.ctypes.c_uint(0)
    _lib.call("fo_median_timeouts", _lib.ctypes.byref(c))
    return int(c.value)


def register_with_flaggems():
    """Registers median with FlagGems when it is installed (median.py:363-372)."""
    try:
        import flag_gems
        if hasattr(flag_gems, "_C"):
            flag_gems._C.register_op("aten::median", median)
        logger.info("flag-ops: median registered with FlagGems")
    except Exception as e:  # FlagGems absent or API mismatch: nothing to register
        logger.debug("flag-ops: FlagGems registration skipped: %s", e)
