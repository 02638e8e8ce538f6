"""rms_norm — drop-in for operators/rms_norm.py of Flag-Operators.

Same public functions, argument names and defaults as the reference
(operators/rms_norm.py:186-252).  The forward is one sm_100a kernel
(csrc/rms_norm.cu, entry point fo_rms_norm_fwd): each row is read from HBM once
and written once.

Addition: rms_norm_backward(dy, x, inv_rms, normalized_shape, weight) -> (dx, dw),
the backward that the reference's inv_rms output is meant for (its forward
returns it "for backward", rms_norm.py:10-17), as one kernel over the rows
(csrc/rms_norm_bwd.cu, fo_rms_norm_bwd); rms_norm() is differentiable through it.
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


def rms_norm_backward(
    dy: torch.Tensor,
    x: torch.Tensor,
    inv_rms: torch.Tensor,
    normalized_shape,
    weight: torch.Tensor,
):
    """(dx, dw) of y = x * inv_rms * weight, given the forward's inv_rms.

    dx = inv * (dy * w) - x * inv^3 * sum(dy * w * x) / N  (x's dtype)
    dw = sum over rows of dy * x * inv                      (weight's dtype)
    """
    _lib.require_cuda(x, "rms_norm_backward")
    if isinstance(normalized_shape, int):
        normalized_shape = (normalized_shape,)
    N = math.prod(normalized_shape)
    if N <= 0:
        raise ValueError("rms_norm_backward: normalized size must be > 0")
    M = x.numel() // N
    x = x.contiguous()
    dy = dy.to(x.dtype).contiguous()
    if dy.shape != x.shape:
        raise ValueError(f"rms_norm_backward: dy shape {tuple(dy.shape)} != x shape {tuple(x.shape)}")
    w = weight.contiguous().view(-1)
    if w.numel() != N:
        raise ValueError(f"rms_norm_backward: weight has {w.numel()} elements, expected {N}")
    inv = inv_rms.to(torch.float32).contiguous().view(-1)
    if inv.numel() != M:
        raise ValueError(f"rms_norm_backward: inv_rms has {inv.numel()} elements, expected {M}")
    dx = torch.empty_like(x)
    dw = torch.empty(weight.shape, dtype=weight.dtype, device=x.device)
    import ctypes
    nbytes = ctypes.c_int64(0)
    _lib.call("fo_rms_norm_bwd_workspace_bytes", M, N, ctypes.byref(nbytes))
    ws = torch.empty(max(nbytes.value, 1), dtype=torch.uint8, device=x.device)
    _lib.call("fo_rms_norm_bwd", _lib.ptr(dy), _lib.ptr(x), _lib.ptr(w), _lib.ptr(inv),
              _lib.ptr(dx), _lib.ptr(dw), M, N, _lib.dtype_code(x.dtype),
              _lib.dtype_code(w.dtype), _lib.ptr(ws), nbytes.value, _lib.stream_of(x))
    return dx, dw


class _RmsNorm(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, normalized_shape, weight, eps):
        y, inv_rms = rms_norm_forward(x, normalized_shape, weight, eps)
        ctx.save_for_backward(x, weight, inv_rms)
        ctx.normalized_shape = normalized_shape
        return y

    @staticmethod
    def backward(ctx, dy):
        x, weight, inv_rms = ctx.saved_tensors
        dx, dw = rms_norm_backward(dy, x, inv_rms, ctx.normalized_shape, weight)
        return (dx if ctx.needs_input_grad[0] else None, None,
                dw if ctx.needs_input_grad[2] else None, None)


def rms_norm(
    x: torch.Tensor,
    normalized_shape,
    weight: torch.Tensor,
    eps: float = 1e-5,
) -> torch.Tensor:
    """Returns only y (operators/rms_norm.py:231-240); differentiable in x and weight."""
    if torch.is_grad_enabled() and (x.requires_grad or weight.requires_grad):
        _lib.require_cuda(x, "rms_norm")
        return _RmsNorm.apply(x, normalized_shape, weight, eps)
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
