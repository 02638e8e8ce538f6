"""rms_norm — drop-in for operators/rms_norm.py of Flag-Operators.

Same public functions, argument names and defaults as the reference
(operators/rms_norm.py:186-252).  The forward is one sm_100a kernel
(csrc/rms_norm.cu, entry point fo_rms_norm_fwd): each row is read from HBM once
and written once.
"""
from __future__ import annotations

import logging
import math

import torch

from . import _lib

logger = logging.getLogger(__name__)


def rms_norm_forward(
    x: torch.Tensor,
    normalized_shape,
    weight: torch.Tensor,
    eps: float = 1e-5,
):
    """Returns (y, inv_rms); API of rms_norm_forward, operators/rms_norm.py:186-228.

    x: [..., *normalized_shape]; weight: [*normalized_shape];
    y has x's dtype and shape, inv_rms is fp32 [M] with M = numel / prod(normalized_shape).
    """
    logger.debug("FLAG-OPS RMS_NORM FORWARD")
    _lib.require_cuda(x, "rms_norm_forward")
    if isinstance(normalized_shape, int):
        normalized_shape = (normalized_shape,)
    N = math.prod(normalized_shape)
    M = x.numel() // N if N > 0 else 0

    x = x.contiguous()
    weight = weight.contiguous().view(-1)
    if weight.numel() != N:
        raise ValueError(f"rms_norm: weight has {weight.numel()} elements, expected {N}")
    if weight.device != x.device:
        raise ValueError("rms_norm: weight must be on the same device as x")
    y = torch.empty_like(x)
    inv_rms = torch.empty(M, dtype=torch.float32, device=x.device)
    if M == 0:
        return y, inv_rms
    _lib.call("fo_rms_norm_fwd", _lib.ptr(x), _lib.ptr(weight), _lib.ptr(y), _lib.ptr(inv_rms),
              M, N, float(eps), _lib.dtype_code(x.dtype), _lib.dtype_code(weight.dtype),
              _lib.stream_of(x))
    return y, inv_rms


def rms_norm(
    x: torch.Tensor,
    normalized_shape,
    weight: torch.Tensor,
    eps: float = 1e-5,
) -> torch.Tensor:
    """Returns only y (operators/rms_norm.py:231-240)."""
    y, _ = rms_norm_forward(x, normalized_shape, weight, eps)
    return y


def rms_norm_out(
    result: torch.Tensor,
    x: torch.Tensor,
    normalized_shape,
    weight: torch.Tensor,
    eps: float = 1e-5,
) -> torch.Tensor:
    """Writes y into `result` (operators/rms_norm.py:242-252).

    When `result` is contiguous with x's dtype and shape the kernel writes into it
    directly (no extra copy pass); otherwise y is computed and copied.
    """
    _lib.require_cuda(x, "rms_norm_out")
    if isinstance(normalized_shape, int):
        normalized_shape = (normalized_shape,)
    N = math.prod(normalized_shape)
    if (result.is_cuda and result.is_contiguous() and result.dtype == x.dtype
            and result.shape == x.shape and result.device == x.device and N > 0
            and result.data_ptr() != x.data_ptr()):
        xc = x.contiguous()
        w = weight.contiguous().view(-1)
        if w.numel() != N:
            raise ValueError(f"rms_norm: weight has {w.numel()} elements, expected {N}")
        M = xc.numel() // N
        if M > 0:
            inv_rms = torch.empty(M, dtype=torch.float32, device=x.device)
            _lib.call("fo_rms_norm_fwd", _lib.ptr(xc), _lib.ptr(w), _lib.ptr(result),
                      _lib.ptr(inv_rms), M, N, float(eps), _lib.dtype_code(xc.dtype),
                      _lib.dtype_code(w.dtype), _lib.stream_of(xc))
        return result
    y, _ = rms_norm_forward(x, normalized_shape, weight, eps)
    result.copy_(y)
    return result
