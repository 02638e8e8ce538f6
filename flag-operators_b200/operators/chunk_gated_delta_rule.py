"""chunk_gated_delta_rule — drop-in for operators/chunk_gated_delta_rule.py of Flag-Operators.

    chunk_gated_delta_rule(q, k, v, beta, g) -> o
    h_t = g_t h_{t-1} + beta_t (v_t - h_{t-1} k_t) k_t^T ,  o_t = h_t q_t

q, k, v: [B, H, L, D] with D in {16, 32, 64, 128}; beta, g: [B, H, L]; o has q's
dtype, the state is fp32 (as the reference, chunk_gated_delta_rule.py:208-268).
Keyword-only extensions (defaults keep the reference behaviour):
  initial_state=None   fp32 [B, H, D, D] state before the first token
  output_final_state=False   also return the fp32 final state: (o, h_T)

Kernels: bf16/fp16 inputs run the chunked tensor-core kernels for every D
(csrc/delta_rule_tc.cu: chunks of 64 tokens, seven tcgen05 GEMMs per chunk,
fp32 state in TMEM, fp16 operand tiles; D < 128 as D = 128 with zero channels);
a head whose fp16 operands would leave the fp16 range is recomputed in the same
call by the fp32 per-step kernel, so finite inputs give finite outputs.  fp32
inputs run the per-step kernel (csrc/delta_rule_step.cu).  _ref_forward is kept importable, as the reference's
tests import it; it is the reference's sequential fp32 loop on CPU tensors.

Backward: when autograd needs a gradient of q, k, v, beta, g or initial_state,
the call goes through an autograd Function whose backward is the fp32 CUDA-core
kernel of csrc/delta_rule_bwd.cu (fo_gdr_bwd).  Its gradients are those torch
autograd gives through the reference's CPU loop (the reference itself has no
backward).  Without a gradient to compute, nothing is saved and the forward
runs as before.
"""
from __future__ import annotations

import ctypes
import logging

import torch
from torch.autograd.function import once_differentiable

from . import _lib

logger = logging.getLogger(__name__)


def _check_inputs(q, k, v, beta, g):
    """The reference's shape checks (chunk_gated_delta_rule.py:198-205)."""
    B, H, L, D = q.shape
    assert k.shape == q.shape, f"k shape {k.shape} != q shape {q.shape}"
    assert v.shape == q.shape, f"v shape {v.shape} != q shape {q.shape}"
    assert beta.shape == (B, H, L), f"beta shape {beta.shape}, expected ({B},{H},{L})"
    assert g.shape == (B, H, L), f"g shape {g.shape}, expected ({B},{H},{L})"
    assert D in (16, 32, 64, 128), f"D={D} not in supported set {{16,32,64,128}}"
    return B, H, L, D


def _forward(q, k, v, beta, g, h0, output_final_state):
    """o (and the fp32 final state) through fo_gdr_fwd; inputs already checked."""
    B, H, L, D = q.shape
    o = torch.empty_like(q)
    hT = torch.empty(B, H, D, D, dtype=torch.float32, device=q.device) \
        if output_final_state else None
    nbytes = ctypes.c_int64(0)
    _lib.call("fo_gdr_workspace_bytes", B, H, L, D, _lib.dtype_code(q.dtype),
              ctypes.byref(nbytes))
    ws = torch.empty(nbytes.value, dtype=torch.uint8, device=q.device) if nbytes.value else None
    _lib.call("fo_gdr_fwd", _lib.ptr(q), _lib.ptr(k), _lib.ptr(v), _lib.ptr(beta), _lib.ptr(g),
              _lib.ptr(h0), _lib.ptr(o), _lib.ptr(hT), B, H, L, D, _lib.dtype_code(q.dtype),
              _lib.dtype_code(beta.dtype), _lib.ptr(ws), nbytes.value, _lib.stream_of(q))
    return o, hT


def _backward(q, k, v, beta, g, h0, do, dhT, need_dh0):
    """(dq, dk, dv, dbeta, dg, dh0) through fo_gdr_bwd; do / dhT may be None."""
    B, H, L, D = q.shape
    do = torch.zeros_like(q) if do is None else do.to(q.dtype).contiguous()
    if dhT is not None:
        dhT = dhT.to(torch.float32).contiguous()
    dq, dk, dv = torch.empty_like(q), torch.empty_like(k), torch.empty_like(v)
    dbeta, dg = torch.empty_like(beta), torch.empty_like(beta)
    dh0 = torch.empty(B, H, D, D, dtype=torch.float32, device=q.device) if need_dh0 else None
    nbytes = ctypes.c_int64(0)
    _lib.call("fo_gdr_bwd_workspace_bytes", B, H, L, D, ctypes.byref(nbytes))
    ws = torch.empty(nbytes.value, dtype=torch.uint8, device=q.device) if nbytes.value else None
    _lib.call("fo_gdr_bwd", _lib.ptr(q), _lib.ptr(k), _lib.ptr(v), _lib.ptr(beta), _lib.ptr(g),
              _lib.ptr(h0), _lib.ptr(do), _lib.ptr(dhT), _lib.ptr(dq), _lib.ptr(dk),
              _lib.ptr(dv), _lib.ptr(dbeta), _lib.ptr(dg), _lib.ptr(dh0), B, H, L, D,
              _lib.dtype_code(q.dtype), _lib.dtype_code(beta.dtype), _lib.ptr(ws), nbytes.value,
              _lib.stream_of(q))
    return dq, dk, dv, dbeta, dg, dh0


class _GatedDeltaRule(torch.autograd.Function):
    """Forward through fo_gdr_fwd, backward through fo_gdr_bwd (inputs are saved;
    the backward recomputes the states from them)."""

    @staticmethod
    def forward(ctx, q, k, v, beta, g, h0, output_final_state):
        o, hT = _forward(q, k, v, beta, g, h0, output_final_state)
        ctx.save_for_backward(q, k, v, beta, g, h0)
        ctx.set_materialize_grads(False)
        if output_final_state:
            return o, hT
        return o

    @staticmethod
    @once_differentiable
    def backward(ctx, do, dhT=None):
        # first derivatives only: a double backward raises instead of returning
        # wrong second derivatives
        q, k, v, beta, g, h0 = ctx.saved_tensors
        dq, dk, dv, dbeta, dg, dh0 = _backward(q, k, v, beta, g, h0, do, dhT,
                                               h0 is not None and ctx.needs_input_grad[5])
        return dq, dk, dv, dbeta, dg, dh0, None


def chunk_gated_delta_rule(
    q: torch.Tensor,
    k: torch.Tensor,
    v: torch.Tensor,
    beta: torch.Tensor,
    g: torch.Tensor,
    *,
    initial_state: torch.Tensor | None = None,
    output_final_state: bool = False,
):
    """Gated delta rule forward (chunk_gated_delta_rule.py:208-268), differentiable."""
    logger.debug("FLAG-OPS CHUNK_GATED_DELTA_RULE")
    _lib.require_cuda(q, "chunk_gated_delta_rule")
    B, H, L, D = _check_inputs(q, k, v, beta, g)
    if not (k.dtype == q.dtype and v.dtype == q.dtype):
        raise TypeError("chunk_gated_delta_rule: q, k and v must share a dtype")
    if beta.dtype != g.dtype:
        g = g.to(beta.dtype)
    q, k, v = q.contiguous(), k.contiguous(), v.contiguous()
    beta, g = beta.contiguous(), g.contiguous()
    h0 = None
    if initial_state is not None:
        assert initial_state.shape == (B, H, D, D), (
            f"initial_state shape {tuple(initial_state.shape)}, expected ({B},{H},{D},{D})")
        h0 = initial_state.to(device=q.device, dtype=torch.float32).contiguous()
    if torch.is_grad_enabled() and any(
            t is not None and t.requires_grad for t in (q, k, v, beta, g, h0)):
        return _GatedDeltaRule.apply(q, k, v, beta, g, h0, output_final_state)
    o, hT = _forward(q, k, v, beta, g, h0, output_final_state)
    if output_final_state:
        return o, hT
    return o


def _ref_forward(q, k, v, beta, g):
    """The reference's sequential loop (chunk_gated_delta_rule.py:275-310), CPU/any device.

    Kept because the reference's tests import it; it is not used by the kernels.
    """
    B, H, L, D = q.shape
    dtype = q.dtype
    h = torch.zeros(B, H, D, D, dtype=torch.float32, device=q.device)
    o = torch.empty_like(q)
    for t in range(L):
        q_t = q[:, :, t, :].float()
        k_t = k[:, :, t, :].float()
        v_t = v[:, :, t, :].float()
        beta_t = beta[:, :, t]
        g_t = g[:, :, t]
        residual = (h @ k_t.unsqueeze(-1)).squeeze(-1)
        delta = v_t - residual
        h = (g_t[:, :, None, None] * h
             + beta_t[:, :, None, None] * (delta.unsqueeze(-1) * k_t.unsqueeze(-2)))
        o[:, :, t, :] = (h @ q_t.unsqueeze(-1)).squeeze(-1).to(dtype)
    return o


def timeouts() -> int:
    """Tensor-core waits that ran out of polls since load (0 in a healthy run)."""
    c = _lib.ctypes.c_uint(0)
    _lib.call("fo_gdr_timeouts", _lib.ctypes.byref(c))
    return int(c.value)
