"""CPU restatement of the reference's CPU path (test infrastructure only).

Each function names the reference lines it restates (paths inside the
iamsuperfly/Flag-Operators project).  The reference's CPU branch is plain torch
on CPU tensors; the restatement keeps exactly that arithmetic so its outputs are
the reference's outputs.  `median_dim_np` is an independent numpy statement of
torch's median index rule, used to pin the semantics the kernels must match.
"""
from __future__ import annotations

import math

import numpy as np
import torch
import torch.nn.functional as F


def _cpu(t):
    return t.detach().cpu() if isinstance(t, torch.Tensor) else t


# ---------------------------------------------------------------------------
# rms_norm — operators/rms_norm.py:201-216 (CPU fallback branch)
# ---------------------------------------------------------------------------
def rms_norm_forward(x, normalized_shape, weight, eps=1e-5):
    """(y, inv_rms) exactly as rms_norm.py:209-216 computes them on CPU."""
    x = _cpu(x)
    weight = _cpu(weight)
    if isinstance(normalized_shape, int):
        normalized_shape = (normalized_shape,)
    N = math.prod(normalized_shape)          # rms_norm.py:201
    M = x.numel() // N                       # rms_norm.py:202
    x = x.contiguous()                       # rms_norm.py:204
    weight = weight.contiguous().view(-1)    # rms_norm.py:205
    y = torch.empty_like(x)                  # rms_norm.py:206
    inv_rms = torch.empty(M, dtype=torch.float32)
    xf = x.float().view(M, N)                                    # rms_norm.py:211
    rms = torch.sqrt((xf * xf).mean(dim=-1, keepdim=True) + eps)  # rms_norm.py:212
    yf = (xf / rms) * weight.float()                             # rms_norm.py:213
    y.copy_(yf.view_as(x))                                       # rms_norm.py:214
    inv_rms.copy_(1.0 / rms.squeeze(-1))                         # rms_norm.py:215
    return y, inv_rms


def rms_norm_backward(dy, x, normalized_shape, weight, eps=1e-5):
    """(dx, dw) of the CPU forward of rms_norm.py:211-213 by autograd, in fp32.

    The reference has no backward of its own; its forward returns inv_rms for a
    backward (rms_norm.py:10-17), whose result is the gradient of this formula.
    """
    x = _cpu(x).float().clone().requires_grad_(True)
    w = _cpu(weight).float().clone().requires_grad_(True)
    if isinstance(normalized_shape, int):
        normalized_shape = (normalized_shape,)
    N = math.prod(normalized_shape)
    xf = x.view(-1, N)
    rms = torch.sqrt((xf * xf).mean(dim=-1, keepdim=True) + eps)
    y = (xf / rms) * w.view(-1)
    y.backward(_cpu(dy).float().view(-1, N))
    return x.grad.detach(), w.grad.detach()


# ---------------------------------------------------------------------------
# median — operators/median.py:348-352 (CPU branch: torch.median)
# ---------------------------------------------------------------------------
def median(inp, dim=None, keepdim=False):
    inp = _cpu(inp)
    if dim is None:
        return torch.median(inp)                                  # median.py:350-351
    return torch.median(inp, dim=dim, keepdim=keepdim)            # median.py:352


def median_dim_np(x2d: np.ndarray):
    """Independent statement of torch CPU's median-along-dim rule for a 2-D array.

    values, indices of each row: k = (N-1)//2; the index is the k-th entry of a
    stable ascending sort (ties keep index order, -0.0 == +0.0); a row holding a
    NaN yields NaN and the index of its first NaN.
    """
    x2d = np.asarray(x2d)
    M, N = x2d.shape
    k = (N - 1) // 2
    order = np.argsort(x2d, axis=1, kind="stable")
    idx = order[:, k].astype(np.int64)
    isnan = np.isnan(x2d) if np.issubdtype(x2d.dtype, np.floating) else np.zeros_like(x2d, bool)
    has_nan = isnan.any(axis=1)
    if has_nan.any():
        first_nan = np.argmax(isnan, axis=1)
        idx = np.where(has_nan, first_nan, idx)
    vals = x2d[np.arange(M), idx]
    return vals, idx


# ---------------------------------------------------------------------------
# scatter_reduce — operators/scatter_reduce.py:397-398, 427-429, 457-459
# ---------------------------------------------------------------------------
def scatter_reduce_(inp, dim, index, src, reduce, *, include_self=True):
    return _cpu(inp).clone().scatter_reduce_(dim, _cpu(index), _cpu(src), reduce,
                                             include_self=include_self)


def scatter_reduce(inp, dim, index, src, reduce, *, include_self=True):
    return torch.scatter_reduce(_cpu(inp), dim, _cpu(index), _cpu(src), reduce,
                                include_self=include_self)


def scatter_reduce_out(out, inp, dim, index, src, reduce, *, include_self=True):
    out_c = torch.empty_like(_cpu(out))
    return torch.scatter_reduce(_cpu(inp), dim, _cpu(index), _cpu(src), reduce,
                                include_self=include_self, out=out_c)


def scatter_reduce_scale(inp, dim, index, src, include_self=True):
    """Per-cell (sum of |terms|, number of terms) in float64, for tolerances.

    A float sum's rounding error is bounded by a multiple of the sum of the
    magnitudes of its terms, so parity of float sum/mean is checked against
    rtol * this scale rather than rtol * |result|.
    """
    inp = _cpu(inp).double()
    index = _cpu(index)
    src = _cpu(src).double()
    base_abs = inp.abs() if include_self else torch.zeros_like(inp)
    base_cnt = torch.ones_like(inp) if include_self else torch.zeros_like(inp)
    scale = base_abs.scatter_add(dim, index, src.abs()[tuple(slice(0, s) for s in index.shape)])
    cnt = base_cnt.scatter_add(dim, index, torch.ones(index.shape, dtype=torch.float64))
    return scale, cnt


# ---------------------------------------------------------------------------
# fused_cross_entropy — operators/fused_cross_entropy.py:327-331 (F.cross_entropy)
# ---------------------------------------------------------------------------
def fused_cross_entropy(logits, target, reduction="mean", ignore_index=-100, label_smoothing=0.0):
    return F.cross_entropy(_cpu(logits), _cpu(target), reduction=reduction,
                           ignore_index=ignore_index, label_smoothing=label_smoothing)


def fused_cross_entropy_grad(logits, target, reduction="mean", ignore_index=-100,
                             label_smoothing=0.0, grad_output=None):
    """(loss, dlogits) of the CPU branch via autograd (fused_cross_entropy.py:327-331)."""
    lg = _cpu(logits).clone().requires_grad_(True)
    loss = F.cross_entropy(lg, _cpu(target), reduction=reduction, ignore_index=ignore_index,
                           label_smoothing=label_smoothing)
    go = torch.ones_like(loss) if grad_output is None else _cpu(grad_output).to(loss.dtype)
    loss.backward(go)
    return loss.detach(), lg.grad.detach()


# ---------------------------------------------------------------------------
# chunk_gated_delta_rule — _ref_forward, operators/chunk_gated_delta_rule.py:275-310
# ---------------------------------------------------------------------------
def delta_rule_forward(q, k, v, beta, g, initial_state=None, output_final_state=False):
    """Sequential fp32 recurrence of _ref_forward (chunk_gated_delta_rule.py:286-310).

    h_t = g_t h_{t-1} + beta_t (v_t - h_{t-1} k_t) k_t^T ;  o_t = h_t q_t (cast to q's dtype).
    Extends the reference with an optional fp32 initial state [B,H,D,D] and
    returns (o, h_T) when output_final_state is set.
    """
    q, k, v, beta, g = (_cpu(t) for t in (q, k, v, beta, g))
    B, H, L, D = q.shape
    dtype = q.dtype
    if initial_state is None:
        h = torch.zeros(B, H, D, D, dtype=torch.float32)                 # :288
    else:
        h = _cpu(initial_state).float().clone()
    o = torch.empty_like(q)                                               # :289
    for t in range(L):                                                    # :291
        q_t = q[:, :, t, :].float()                                       # :292
        k_t = k[:, :, t, :].float()                                       # :293
        v_t = v[:, :, t, :].float()                                       # :294
        beta_t = beta[:, :, t]                                            # :295
        g_t = g[:, :, t]                                                  # :296
        residual = (h @ k_t.unsqueeze(-1)).squeeze(-1)                    # :299
        delta = v_t - residual                                            # :300
        h = (g_t[:, :, None, None] * h                                    # :303-305
             + beta_t[:, :, None, None] * (delta.unsqueeze(-1) * k_t.unsqueeze(-2)))
        o[:, :, t, :] = (h @ q_t.unsqueeze(-1)).squeeze(-1).to(dtype)     # :308
    if output_final_state:
        return o, h
    return o


def delta_rule_grads(q, k, v, beta, g, do, initial_state=None, dhT=None):
    """Gradients of the reference's CPU recurrence by torch autograd.

    The reference's CPU branch (_ref_forward, chunk_gated_delta_rule.py:286-310) is
    plain differentiable torch; the reference ships no backward of its own, so the
    gradients it defines are autograd's through that loop.  The loop below is the
    same statement (fp32 state, inputs read as fp32, gates promoted against the
    fp32 state), with o_t kept in fp32 (the cast to q's dtype at :308 has an
    identity backward).  Loss = sum(o * do) + sum(h_T * dhT); returns fp32
    gradients {q, k, v, beta, g, initial_state}.
    """
    leaves = [_cpu(t).float().clone().requires_grad_(True) for t in (q, k, v, beta, g)]
    qf, kf, vf, bf, gf = leaves
    B, H, L, D = qf.shape
    if initial_state is None:
        h0 = torch.zeros(B, H, D, D, dtype=torch.float32, requires_grad=True)
    else:
        h0 = _cpu(initial_state).float().clone().requires_grad_(True)
    h = h0
    outs = []
    for t in range(L):
        k_t = kf[:, :, t, :]
        delta = vf[:, :, t, :] - (h @ k_t.unsqueeze(-1)).squeeze(-1)
        h = (gf[:, :, t, None, None] * h
             + bf[:, :, t, None, None] * (delta.unsqueeze(-1) * k_t.unsqueeze(-2)))
        outs.append((h @ qf[:, :, t, :].unsqueeze(-1)).squeeze(-1))
    loss = torch.zeros((), dtype=torch.float32)
    if L:
        loss = loss + (torch.stack(outs, dim=2) * _cpu(do).float()).sum()
    if dhT is not None:
        loss = loss + (h * _cpu(dhT).float()).sum()
    if loss.requires_grad:
        loss.backward()
    names = ("q", "k", "v", "beta", "g")
    res = {n: (x.grad if x.grad is not None else torch.zeros_like(x)) for n, x in zip(names, leaves)}
    res["initial_state"] = h0.grad if h0.grad is not None else torch.zeros_like(h0)
    return res


def delta_rule_backward(q, k, v, beta, g, do, initial_state=None, dhT=None):
    """The per-step reverse recurrence the CUDA backward implements, in float64.

    With h_{t-1} the state before step t, delta_t = v_t - h_{t-1} k_t and G the
    gradient of the loss with respect to h_t (do_t q_t^T plus what flows back from
    h_{t+1}), differentiating h_t = g_t h_{t-1} + beta_t delta_t k_t^T and
    o_t = h_t q_t gives, per step in reverse:
      gk = G k_t;  dv_t = beta_t gk;  dbeta_t = gk . delta_t;  dg_t = <G, h_{t-1}>
      dq_t = h_t^T do_t = g_t h_{t-1}^T do_t + beta_t (delta_t . do_t) k_t
      dk_t = beta_t (G^T delta_t - h_{t-1}^T gk)
      G <- g_t G - beta_t gk k_t^T          (the gradient with respect to h_{t-1})
    and the initial state's gradient is the final G.  Checked against
    delta_rule_grads (autograd) by the CPU tests.
    """
    q, k, v, beta, g, do = (_cpu(t).double() for t in (q, k, v, beta, g, do))
    B, H, L, D = q.shape
    h = (torch.zeros(B, H, D, D, dtype=torch.float64) if initial_state is None
         else _cpu(initial_state).double().clone())
    hs = []
    for t in range(L):
        hs.append(h)
        k_t = k[:, :, t]
        delta = v[:, :, t] - (h @ k_t[..., None])[..., 0]
        h = g[:, :, t, None, None] * h + beta[:, :, t, None, None] * (delta[..., None]
                                                                         * k_t[..., None, :])
    G = (torch.zeros(B, H, D, D, dtype=torch.float64) if dhT is None
         else _cpu(dhT).double().clone())
    dq, dk, dv = torch.zeros_like(q), torch.zeros_like(k), torch.zeros_like(v)
    dbeta, dg = torch.zeros_like(beta), torch.zeros_like(g)
    for t in reversed(range(L)):
        hp, k_t, q_t, do_t = hs[t], k[:, :, t], q[:, :, t], do[:, :, t]
        b_t, g_t = beta[:, :, t, None], g[:, :, t, None]
        G = G + do_t[..., None] * q_t[..., None, :]
        gk = (G @ k_t[..., None])[..., 0]
        delta = v[:, :, t] - (hp @ k_t[..., None])[..., 0]
        dv[:, :, t] = b_t * gk
        dbeta[:, :, t] = (gk * delta).sum(-1)
        dg[:, :, t] = (G * hp).sum((-1, -2))
        dq[:, :, t] = (g_t * (hp.transpose(-1, -2) @ do_t[..., None])[..., 0]
                       + b_t * (delta * do_t).sum(-1, keepdim=True) * k_t)
        dk[:, :, t] = b_t * ((G.transpose(-1, -2) @ delta[..., None])[..., 0]
                             - (hp.transpose(-1, -2) @ gk[..., None])[..., 0])
        G = g_t[..., None] * G - b_t[..., None] * gk[..., None] * k_t[..., None, :]
    return {"q": dq, "k": dk, "v": dv, "beta": dbeta, "g": dg, "initial_state": G}


def delta_rule_backward_chunked(q, k, v, beta, g, do, initial_state=None, dhT=None, C=16):
    """The chunked backward (the form a tensor-core kernel would take), float64.

    Forward of a chunk with entry state S [Dv, Dk], tokens t = 0..n-1, in-chunk
    gate products gam_t = g_0 ... g_t (gam_{-1} = 1), ratio(t, s) = gam_t / gam_s:
      A[t,s] = ratio(t-1,s) beta_s k_t.k_s (s < t),  T = (I + A)^-1
      R = V - diag(gam_{t-1}) K S^T,  U = T R
      P[t,s] = ratio(t,s) beta_s q_t.k_s (s <= t),  O = diag(gam_t) Q S^T + P U
      Kt[s] = ratio(n-1,s) beta_s k_s,  S' = gam_{n-1} S + U^T Kt
    Backward of the chunk, given dO and dS' (the transposes of those products):
      dU = P^T dO + Kt dS'^T;  dP = dO U^T (s <= t);  dKt = U dS'
      dR = T^T dU;  dT = dU R^T;  dA = -T^T dT T^T (s < t);  dV = dR
      dS = dO^T diag(gam) Q + gam_{n-1} dS' - dR^T diag(gam_{t-1}) K
      dQ = diag(gam) dO S + (dP o ratio o beta) K
      dK = -diag(gam_{t-1}) dR S + (dA o ratio' o beta) K + (dA o ratio' o beta)^T K
           + (dP o ratio o beta)^T Q + diag(ratio(n-1,.) beta) dKt
    and dbeta, dgam from the same products; dg_r = sum_{t >= r} dgam_t gam_t / g_r
    inside the chunk.  dS is carried to the previous chunk as its dS'.  Gates must
    be nonzero (the ratios are formed by division).  Checked against
    delta_rule_grads (autograd) by the CPU tests.
    """
    q, k, v, beta, g, do = (_cpu(t).double() for t in (q, k, v, beta, g, do))
    B, H, L, D = q.shape
    S = (torch.zeros(B, H, D, D, dtype=torch.float64) if initial_state is None
         else _cpu(initial_state).double().clone())
    nch = (L + C - 1) // C
    entry = []
    chunks = []
    for c in range(nch):
        t0, t1 = c * C, min(L, (c + 1) * C)
        Q, K, V = q[:, :, t0:t1], k[:, :, t0:t1], v[:, :, t0:t1]
        bt, gt = beta[:, :, t0:t1], g[:, :, t0:t1]
        n = t1 - t0
        gam = torch.cumprod(gt, dim=-1)                                   # [B,H,n]
        gm1 = torch.cat([torch.ones_like(gam[..., :1]), gam[..., :-1]], -1)
        low = torch.tril(torch.ones(n, n, dtype=torch.float64), -1)
        lowd = torch.tril(torch.ones(n, n, dtype=torch.float64))
        rA = gm1[..., :, None] / gam[..., None, :]                        # ratio(t-1, s)
        rP = gam[..., :, None] / gam[..., None, :]                        # ratio(t, s)
        A = low * rA * bt[..., None, :] * (K @ K.transpose(-1, -2))
        T = torch.linalg.inv(torch.eye(n, dtype=torch.float64) + A)
        R = V - gm1[..., None] * (K @ S.transpose(-1, -2))
        U = T @ R
        P = lowd * rP * bt[..., None, :] * (Q @ K.transpose(-1, -2))
        rK = gam[..., -1:] / gam                                          # ratio(n-1, s)
        Kt = (rK * bt)[..., None] * K
        entry.append(S)
        chunks.append((t0, t1, Q, K, V, bt, gt, gam, gm1, low, lowd, rA, rP, T, R, U, P, rK, Kt))
        S = gam[..., -1, None, None] * S + U.transpose(-1, -2) @ Kt
    dS_next = (torch.zeros(B, H, D, D, dtype=torch.float64) if dhT is None
               else _cpu(dhT).double().clone())
    dq, dk, dv = torch.zeros_like(q), torch.zeros_like(k), torch.zeros_like(v)
    dbeta, dg = torch.zeros_like(beta), torch.zeros_like(g)
    for c in reversed(range(nch)):
        (t0, t1, Q, K, V, bt, gt, gam, gm1, low, lowd, rA, rP, T, R, U, P, rK, Kt) = chunks[c]
        S = entry[c]
        dO = do[:, :, t0:t1]
        Sk = K @ S.transpose(-1, -2)                                      # rows S k_t
        Sq = Q @ S.transpose(-1, -2)                                      # rows S q_t
        dU = P.transpose(-1, -2) @ dO + Kt @ dS_next.transpose(-1, -2)
        dP = lowd * (dO @ U.transpose(-1, -2))
        dKt = U @ dS_next
        dR = T.transpose(-1, -2) @ dU
        dT = dU @ R.transpose(-1, -2)
        dA = low * -(T.transpose(-1, -2) @ dT @ T.transpose(-1, -2))
        dS = (dO.transpose(-1, -2) @ (gam[..., None] * Q) + gam[..., -1, None, None] * dS_next
              - dR.transpose(-1, -2) @ (gm1[..., None] * K))
        MP = dP * rP * bt[..., None, :]
        MA = dA * rA * bt[..., None, :]
        dq[:, :, t0:t1] = gam[..., None] * (dO @ S) + MP @ K
        dk[:, :, t0:t1] = (-gm1[..., None] * (dR @ S) + MA @ K + MA.transpose(-1, -2) @ K
                           + MP.transpose(-1, -2) @ Q + (rK * bt)[..., None] * dKt)
        dv[:, :, t0:t1] = dR
        KK, QK = K @ K.transpose(-1, -2), Q @ K.transpose(-1, -2)
        dbeta[:, :, t0:t1] = ((dA * rA * KK).sum(-2) + (dP * rP * QK).sum(-2)
                              + rK * (dKt * K).sum(-1))
        # gradients with respect to the in-chunk gate products gam
        GA = dA * bt[..., None, :] * KK                                   # d/d ratio(t-1, s)
        GP = dP * bt[..., None, :] * QK                                   # d/d ratio(t, s)
        GK = bt * (dKt * K).sum(-1)                                       # d/d ratio(n-1, s)
        dgam = (dO * Sq).sum(-1)                                          # O direct term
        dgam = dgam + (GP / gam[..., None, :]).sum(-1)
        dgam = dgam - (GP * gam[..., :, None]).sum(-2) / gam ** 2
        dgam = dgam - (GA * gm1[..., :, None]).sum(-2) / gam ** 2
        dgm1 = (GA / gam[..., None, :]).sum(-1) - (dR * Sk).sum(-1)       # d/d gam_{t-1}
        dgam[..., :-1] = dgam[..., :-1] + dgm1[..., 1:]
        dgam[..., -1] = (dgam[..., -1] + (dS_next * S).sum((-1, -2))
                         + (GK / gam).sum(-1))
        dgam = dgam - GK * gam[..., -1:] / gam ** 2
        # gam_t = g_0 ... g_t: dg_r = sum_{t >= r} dgam_t gam_t / g_r
        suffix = torch.flip(torch.cumsum(torch.flip(dgam * gam, [-1]), -1), [-1])
        dg[:, :, t0:t1] = suffix / gt
        dS_next = dS
    return {"q": dq, "k": dk, "v": dv, "beta": dbeta, "g": dg, "initial_state": dS_next}


# ---------------------------------------------------------------------------
# vocabulary-sharded cross-entropy: statement of the sharded algorithm on CPU
# (used by the multi-process tests to check the host logic and the combine rule;
# the single-device result it must reproduce is F.cross_entropy above)
# ---------------------------------------------------------------------------
def ce_shard_stats(logits_block, target, v_offset, ignore_index=-100):
    """[B, 4] float64: (row max, sum exp(x - max), target logit if in block else 0, row sum)."""
    x = _cpu(logits_block).double()
    t = _cpu(target)
    m = x.max(dim=1).values
    s = torch.exp(x - m[:, None]).sum(dim=1)
    cols = t - v_offset
    inb = (t != ignore_index) & (cols >= 0) & (cols < x.shape[1])
    xt = torch.where(inb, x.gather(1, cols.clamp(0, x.shape[1] - 1)[:, None]).squeeze(1),
                     torch.zeros_like(m))
    return torch.stack([m, s, xt, x.sum(dim=1)], dim=1)


def ce_shard_combine(all_stats, target, V, ignore_index=-100, label_smoothing=0.0,
                     reduction="mean"):
    """Combines [P, B, 4] block statistics into the loss, as on one device."""
    st = _cpu(all_stats).double()
    t = _cpu(target)
    m = st[:, :, 0].max(dim=0).values
    s = (st[:, :, 1] * torch.exp(st[:, :, 0] - m[None, :])).sum(dim=0)
    lse = m + torch.log(s)
    xt = st[:, :, 2].sum(dim=0)
    rowsum = st[:, :, 3].sum(dim=0)
    valid = t != ignore_index
    e = label_smoothing
    loss = torch.where(valid, lse - (1 - e) * xt - e * rowsum / V, torch.zeros_like(lse))
    if reduction == "none":
        return loss
    if reduction == "sum":
        return loss.sum()
    return loss.sum() / valid.sum()


# ---------------------------------------------------------------------------
# row-sharded cross-entropy: each rank holds a block of the batch's rows; the
# single-device result it must reproduce is F.cross_entropy above
# ---------------------------------------------------------------------------
def ce_rows_partial(logits_rows, target_rows, ignore_index=-100, label_smoothing=0.0):
    """(sum of this block's row losses, number of non-ignored rows), float64."""
    loss = F.cross_entropy(_cpu(logits_rows).double(), _cpu(target_rows), reduction="none",
                           ignore_index=ignore_index, label_smoothing=label_smoothing)
    n = (_cpu(target_rows) != ignore_index).sum()
    return torch.stack([loss.sum(), n.double()])


def ce_rows_combine(partials, reduction="mean"):
    """Combines the [P, 2] per-rank (loss sum, valid rows) into the batch loss."""
    tot = _cpu(partials).double().sum(dim=0)
    return tot[0] / tot[1] if reduction == "mean" else tot[0]
