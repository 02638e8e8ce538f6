"""fused_cross_entropy — drop-in for operators/fused_cross_entropy.py of Flag-Operators.

Public API as the reference (fused_cross_entropy.py:302-380): fused_cross_entropy,
cross_entropy_loss, and the autograd Function _FusedCrossEntropy.  Results follow
torch's F.cross_entropy (the reference's CPU branch): the loss has the logits'
dtype, 'mean' divides by the number of non-ignored rows (NaN if there are none)
and label smoothing is computed inside the kernel.

When the logits require grad, the forward kernel also writes d loss / d logits
for grad_output == 1 while the row is still in L2; backward then only rescales
it in place when grad_output != 1 (a kernel that exits immediately when it is
1).  Forward + backward therefore read the logits from HBM once and write the
gradient once.  The mean divisor is counted on the device: no host sync.

Extension (keyword-only, default keeps the reference behaviour):
``process_group=`` computes the loss of vocabulary-sharded logits: each rank
holds columns [rank*V_local, (rank+1)*V_local) of the [B, V] logits; per-row
(max, sum-exp, target logit, row sum) are all-gathered over NCCL and combined.
``shard="rows"`` instead splits the batch rows over the ranks: the fused
one-read/one-write kernel runs unchanged on each rank's rows, and 'mean' adds two
one-float all-reduces (the valid-row count before the kernel, the loss sum after).
"""
from __future__ import annotations

import ctypes
import logging

import torch

from . import _lib

logger = logging.getLogger(__name__)

_RED = {"none": 0, "mean": 1, "sum": 2}


def _check(logits, target, reduction):
    assert logits.ndim == 2, f"logits must be 2-D [B,V], got shape {logits.shape}"
    assert reduction in ("none", "mean", "sum"), f"Unknown reduction: {reduction}"
    B = logits.shape[0]
    assert target.shape == (B,), f"target shape {target.shape}, expected ({B},)"


class _FusedCrossEntropy(torch.autograd.Function):
    """Autograd Function of the reference (fused_cross_entropy.py:241-295)."""

    @staticmethod
    def forward(ctx, logits, target, reduction, ignore_index, label_smoothing):
        B, V = logits.shape
        assert target.shape == (B,), f"target shape {target.shape}, expected ({B},)"
        dev = logits.device
        target = target.to(torch.int64).contiguous()
        if logits.stride(1) != 1:
            logits = logits.contiguous()
        ld = logits.stride(0) if B > 1 else V
        loss_rows = torch.empty(B, dtype=torch.float32, device=dev)
        lse = torch.empty(B, dtype=torch.float32, device=dev)
        scalar = torch.empty((), dtype=torch.float32, device=dev)
        n_valid = torch.empty(1, dtype=torch.float32, device=dev)
        want_grad = bool(ctx.needs_input_grad[0])
        dlogits = torch.empty((B, V), dtype=logits.dtype, device=dev) if want_grad else None
        _lib.call("fo_ce_fwd", _lib.ptr(logits), _lib.ptr(target), _lib.ptr(loss_rows),
                  _lib.ptr(lse), _lib.ptr(scalar), _lib.ptr(n_valid), _lib.ptr(dlogits),
                  B, V, ld, int(ignore_index), float(label_smoothing), _RED[reduction],
                  _lib.dtype_code(logits.dtype), None, 0, _lib.stream_of(logits))
        out = loss_rows if reduction == "none" else scalar
        ctx.reduction = reduction
        ctx.ignore_index = int(ignore_index)
        ctx.label_smoothing = float(label_smoothing)
        ctx.B, ctx.V, ctx.ld = B, V, ld
        ctx.grad_ready = dlogits is not None
        if dlogits is not None:
            ctx.save_for_backward(logits, target, lse, n_valid, dlogits)
        else:
            ctx.save_for_backward(logits, target, lse, n_valid)
        return out.to(logits.dtype)

    @staticmethod
    def backward(ctx, grad_output):
        saved = ctx.saved_tensors
        logits, target, lse, n_valid = saved[:4]
        B, V = ctx.B, ctx.V
        go = grad_output.contiguous()
        is_vec = 1 if (ctx.reduction == "none" and go.ndim == 1) else 0
        if ctx.grad_ready:
            # gradient for grad_output == 1 was written by the forward pass
            dlogits = saved[4]
            ctx.grad_ready = False
            _lib.call("fo_ce_scale_grad", _lib.ptr(dlogits), _lib.ptr(go),
                      _lib.dtype_code(go.dtype), is_vec, B, V, V,
                      _lib.dtype_code(dlogits.dtype), _lib.stream_of(dlogits))
            return dlogits, None, None, None, None
        dlogits = torch.empty((B, V), dtype=logits.dtype, device=logits.device)
        _lib.call("fo_ce_bwd", _lib.ptr(logits), _lib.ptr(target), _lib.ptr(lse), _lib.ptr(go),
                  _lib.dtype_code(go.dtype), is_vec, _lib.ptr(n_valid), _lib.ptr(dlogits),
                  B, V, ctx.ld, ctx.ignore_index, ctx.label_smoothing, _RED[ctx.reduction],
                  _lib.dtype_code(logits.dtype), _lib.stream_of(logits))
        return dlogits, None, None, None, None


class _PeerUnavailable(RuntimeError):
    """Some rank of the group could not set up or map the exchange regions."""


class _PeerRegions:
    """The NVLink exchange regions of one process group on this rank's device.

    Every rank allocates one region (fo_ce_shard_p2p_region_bytes), zeroes it
    and exports it as a CUDA IPC handle; the handles are exchanged once over
    the group and each rank maps the other ranks' regions, so the fused kernel
    stores its per-row statistics straight into every rank's region.  The
    regions grow (re-exchanged) when a call has more rows than they hold.

    Every rank runs the same collectives whatever fails locally, and the
    outcome is agreed over the group: if any rank could not allocate, export
    or map a region, every rank unmaps what it mapped and raises
    _PeerUnavailable, so no rank is left waiting on another.
    """

    def __init__(self, group, dev, rows):
        import torch.distributed as dist
        self.group, self.dev = group, dev
        self.P, self.rank = dist.get_world_size(group), dist.get_rank(group)
        self.cap = int(rows)
        self.ptrs, self.opened = [], []
        self.region = None
        hb = _lib.load().fo_peer_handle_bytes()
        err = None
        entry = None
        try:
            nbytes = ctypes.c_int64()
            _lib.call("fo_ce_shard_p2p_region_bytes", self.P, self.cap, ctypes.byref(nbytes))
            self.region = torch.zeros(nbytes.value, dtype=torch.uint8, device=dev)
            if dev.type == "cuda":
                torch.cuda.synchronize(dev)  # zeroed before any peer can map and write it
            handle = (ctypes.c_uint8 * hb)()
            off = ctypes.c_int64()
            _lib.call("fo_peer_export", _lib.ptr(self.region), handle, ctypes.byref(off))
            entry = (bytes(handle), off.value)
        except (RuntimeError, ValueError) as e:
            err = e
        entries = [None] * self.P
        dist.all_gather_object(entries, entry, group=group)
        if err is None and any(e is None for e in entries):
            err = RuntimeError("another rank could not export its region")
        if err is None:
            try:
                for p, (h, o) in enumerate(entries):
                    if p == self.rank:
                        self.ptrs.append(self.region.data_ptr())
                        continue
                    out = ctypes.c_void_p()
                    hbuf = (ctypes.c_uint8 * hb).from_buffer_copy(h)
                    _lib.call("fo_peer_open", hbuf, o, ctypes.byref(out))
                    self.ptrs.append(out.value)
                    self.opened.append((out.value, o))
            except (RuntimeError, ValueError) as e:
                err = e
        oks = [None] * self.P
        dist.all_gather_object(oks, err is None, group=group)
        if not all(oks):
            self.close()
            raise _PeerUnavailable(f"NVLink exchange regions unavailable on rank {self.rank}: "
                                   f"{err if err is not None else 'another rank failed'}")
        self.table = (ctypes.c_void_p * self.P)(*self.ptrs)
        self.epoch = 0

    def close(self):
        if self.dev.type == "cuda":
            torch.cuda.synchronize(self.dev)  # no kernel of this rank still uses the mappings
        for ptr_, off in self.opened:
            _lib.call("fo_peer_close", ctypes.c_void_p(ptr_), off)
        self.opened = []


_PEER = {}


def _peer_regions(group, dev, rows):
    """_PeerRegions of the group on dev, or None when the fused NVLink path does
    not apply: fewer than 2 or more than 8 ranks, a backend other than NCCL, ranks
    on more than one host or sharing a GPU, no peer access, or FLAGOPS_CE_P2P=0.
    Every rank reaches the same decision (it is exchanged over the group)."""
    import os
    import socket
    import torch.distributed as dist
    if os.environ.get("FLAGOPS_CE_P2P", "1") == "0":
        return None
    key = (id(group), dev.index)
    st = _PEER.get(key)
    if st is False:
        return None
    if st is not None and st.group is group and st.cap >= rows:
        return st
    P = dist.get_world_size(group)
    if st is None:
        if not (2 <= P <= 8) or dist.get_backend(group) != "nccl":
            _PEER[key] = False
            return None
        infos = [None] * P
        dist.all_gather_object(infos, (socket.gethostname(), dev.index), group=group)
        ok = len({h for h, _ in infos}) == 1 and len({d for _, d in infos}) == P
        for _, d in infos if ok else ():
            c = ctypes.c_int(0)
            _lib.call("fo_peer_can_access", dev.index, d, ctypes.byref(c))
            ok = ok and bool(c.value)
        oks = [None] * P
        dist.all_gather_object(oks, ok, group=group)
        if not all(oks):
            _PEER[key] = False
            return None
    else:
        # more rows than the regions hold: every rank re-allocates at this call
        # (the new regions are zeroed, so the epochs start again at 1)
        st.close()
    try:
        st = _PeerRegions(group, dev, max(int(rows), 1024))
    except _PeerUnavailable:
        _PEER[key] = False  # every rank got here: the all-gather path from now on
        return None
    _PEER[key] = st
    return st


class _ShardedCrossEntropy(torch.autograd.Function):
    """Cross-entropy over vocabulary-sharded logits.

    Ranks on distinct GPUs of one host with peer access: one fused kernel per
    rank (fo_ce_shard_p2p_fwd) computes the row statistics, exchanges them over
    NVLink peer memory and writes the gradient slice in the same pass (one HBM
    read and one write of the block).  Otherwise: per-row statistics, one
    all-gather over the group, a combine kernel, and the gradient recomputed in
    backward.
    """

    @staticmethod
    def forward(ctx, logits, target, reduction, ignore_index, label_smoothing, group, v_offset,
                V):
        import torch.distributed as dist
        B, Vn = logits.shape
        dev = logits.device
        logits = logits if logits.stride(1) == 1 else logits.contiguous()
        ld = logits.stride(0) if B > 1 else Vn
        target = target.to(torch.int64).contiguous()
        P = dist.get_world_size(group)
        ctx.grad_ready = False
        peer = _peer_regions(group, dev, B) if B > 0 else None
        if peer is not None:
            loss_rows = torch.empty(B, dtype=torch.float32, device=dev)
            lse = torch.empty(B, dtype=torch.float32, device=dev)
            scalar = torch.empty((), dtype=torch.float32, device=dev)
            n_valid = torch.empty(1, dtype=torch.float32, device=dev)
            want_grad = bool(ctx.needs_input_grad[0])
            dlogits = torch.empty((B, Vn), dtype=logits.dtype, device=dev) if want_grad else None
            peer.epoch += 1
            _lib.call("fo_ce_shard_p2p_fwd", _lib.ptr(logits), _lib.ptr(target),
                      _lib.ptr(loss_rows), _lib.ptr(lse), _lib.ptr(scalar), _lib.ptr(n_valid),
                      _lib.ptr(dlogits), B, Vn, ld, v_offset, V, int(ignore_index),
                      float(label_smoothing), _RED[reduction], _lib.dtype_code(logits.dtype),
                      peer.table, peer.P, peer.rank, peer.cap, peer.epoch,
                      _lib.stream_of(logits))
            ctx.grad_ready = dlogits is not None
            if dlogits is not None:
                ctx.save_for_backward(logits, target, lse, n_valid, dlogits)
            else:
                ctx.save_for_backward(logits, target, lse, n_valid)
            ctx.args = (reduction, int(ignore_index), float(label_smoothing), v_offset, V, ld)
            out = loss_rows if reduction == "none" else scalar
            return out.to(logits.dtype)
        stats = torch.empty(B, 4, dtype=torch.float32, device=dev)
        _lib.call("fo_ce_shard_stats", _lib.ptr(logits), _lib.ptr(target), _lib.ptr(stats), B,
                  Vn, ld, v_offset, int(ignore_index), _lib.dtype_code(logits.dtype),
                  _lib.stream_of(logits))
        # [P * B, 4]: rank p's rows at [p * B, (p + 1) * B) (the layout NCCL and gloo share)
        all_stats = torch.empty(P * B, 4, dtype=torch.float32, device=dev)
        dist.all_gather_into_tensor(all_stats, stats, group=group)
        loss_rows = torch.empty(B, dtype=torch.float32, device=dev)
        lse = torch.empty(B, dtype=torch.float32, device=dev)
        scalar = torch.empty((), dtype=torch.float32, device=dev)
        n_valid = torch.empty(1, dtype=torch.float32, device=dev)
        _lib.call("fo_ce_shard_combine", _lib.ptr(all_stats), P, _lib.ptr(target),
                  _lib.ptr(loss_rows), _lib.ptr(lse), _lib.ptr(scalar), _lib.ptr(n_valid), B, V,
                  int(ignore_index), float(label_smoothing), _RED[reduction],
                  _lib.stream_of(logits))
        ctx.save_for_backward(logits, target, lse, n_valid)
        ctx.args = (reduction, int(ignore_index), float(label_smoothing), v_offset, V, ld)
        out = loss_rows if reduction == "none" else scalar
        return out.to(logits.dtype)

    @staticmethod
    def backward(ctx, grad_output):
        saved = ctx.saved_tensors
        logits, target, lse, n_valid = saved[:4]
        reduction, ignore_index, ls, v_offset, V, ld = ctx.args
        B, Vn = logits.shape
        go = grad_output.contiguous()
        is_vec = 1 if (reduction == "none" and go.ndim == 1) else 0
        if ctx.grad_ready:
            # the fused kernel wrote the gradient for grad_output == 1
            dlogits = saved[4]
            ctx.grad_ready = False
            _lib.call("fo_ce_scale_grad", _lib.ptr(dlogits), _lib.ptr(go),
                      _lib.dtype_code(go.dtype), is_vec, B, Vn, Vn,
                      _lib.dtype_code(dlogits.dtype), _lib.stream_of(dlogits))
            return dlogits, None, None, None, None, None, None, None
        dlogits = torch.empty((B, Vn), dtype=logits.dtype, device=logits.device)
        _lib.call("fo_ce_shard_bwd", _lib.ptr(logits), _lib.ptr(target), _lib.ptr(lse),
                  _lib.ptr(go), _lib.dtype_code(go.dtype), is_vec, _lib.ptr(n_valid),
                  _lib.ptr(dlogits), B, Vn, ld, v_offset, V, ignore_index, ls, _RED[reduction],
                  _lib.dtype_code(logits.dtype), _lib.stream_of(logits))
        return dlogits, None, None, None, None, None, None, None


class _RowShardedCrossEntropy(torch.autograd.Function):
    """Cross-entropy over a row block of the batch on each rank.

    'mean' needs the batch-wide count of non-ignored rows before the fused
    gradient is written (one all-reduce of a float) and the batch-wide loss sum
    after it (a second all-reduce of a float); 'sum' only the second; 'none'
    no collective at all.
    """

    @staticmethod
    def forward(ctx, logits, target, reduction, ignore_index, label_smoothing, group):
        import torch.distributed as dist
        B, V = logits.shape
        dev = logits.device
        target = target.to(torch.int64).contiguous()
        if logits.stride(1) != 1:
            logits = logits.contiguous()
        ld = logits.stride(0) if B > 1 else V
        st = _lib.stream_of(logits)
        n_valid = torch.empty(1, dtype=torch.float32, device=dev)
        _lib.call("fo_ce_count_valid", _lib.ptr(target), B, int(ignore_index), _lib.ptr(n_valid),
                  st)
        if reduction == "mean":
            dist.all_reduce(n_valid, group=group)
        loss_rows = torch.empty(B, dtype=torch.float32, device=dev)
        lse = torch.empty(B, dtype=torch.float32, device=dev)
        local_sum = torch.empty(1, dtype=torch.float32, device=dev)
        want_grad = bool(ctx.needs_input_grad[0])
        dlogits = torch.empty((B, V), dtype=logits.dtype, device=dev) if want_grad else None
        _lib.call("fo_ce_rows_fwd", _lib.ptr(logits), _lib.ptr(target), _lib.ptr(loss_rows),
                  _lib.ptr(lse), _lib.ptr(local_sum), _lib.ptr(n_valid), _lib.ptr(dlogits), B, V,
                  ld, int(ignore_index), float(label_smoothing), _RED[reduction],
                  _lib.dtype_code(logits.dtype), st)
        if reduction == "none":
            out = loss_rows
        else:
            dist.all_reduce(local_sum, group=group)
            out = (local_sum / n_valid if reduction == "mean" else local_sum).reshape(())
        ctx.reduction = reduction
        ctx.ignore_index = int(ignore_index)
        ctx.label_smoothing = float(label_smoothing)
        ctx.B, ctx.V, ctx.ld = B, V, ld
        ctx.grad_ready = dlogits is not None
        if dlogits is not None:
            ctx.save_for_backward(logits, target, lse, n_valid, dlogits)
        else:
            ctx.save_for_backward(logits, target, lse, n_valid)
        return out.to(logits.dtype)

    @staticmethod
    def backward(ctx, grad_output):
        return _FusedCrossEntropy.backward(ctx, grad_output) + (None,)


def shard_layout(rank: int, world: int, v_local: int, vocab_offset=None, vocab_size=None):
    """(first global column of this rank's block, full vocabulary size).

    Default: equal blocks in rank order, V = v_local * world.  Explicit values
    allow uneven splits; every rank must pass the same vocab_size.
    """
    off = rank * v_local if vocab_offset is None else int(vocab_offset)
    V = v_local * world if vocab_size is None else int(vocab_size)
    if not (0 <= off and off + v_local <= V):
        raise ValueError(f"vocabulary block [{off}, {off + v_local}) outside [0, {V})")
    return off, V


def fused_cross_entropy(
    logits: torch.Tensor,
    target: torch.Tensor,
    reduction: str = "mean",
    ignore_index: int = -100,
    label_smoothing: float = 0.0,
    *,
    process_group=None,
    vocab_offset: int | None = None,
    vocab_size: int | None = None,
    shard: str = "vocab",
) -> torch.Tensor:
    """Fused cross-entropy (fused_cross_entropy.py:302-357).

    logits [B, V], target [B] int64; reduction 'none' | 'mean' | 'sum'.
    With process_group and shard='vocab' (default), logits is this rank's
    [B, V_local] column block; the block starts at vocab_offset (default
    rank * V_local) of a vocabulary of vocab_size columns (default
    V_local * world_size).  With shard='rows', logits [B_local, V] and target
    [B_local] are this rank's rows of the batch: 'none' returns this rank's row
    losses, 'sum' and 'mean' the loss of the whole batch on every rank (mean
    over the non-ignored rows of all ranks), and the gradient of this rank's rows.
    """
    logger.debug("FLAG-OPS FUSED_CROSS_ENTROPY")
    _check(logits, target, reduction)
    _lib.require_cuda(logits, "fused_cross_entropy")
    if not 0.0 <= float(label_smoothing) <= 1.0:
        raise ValueError(f"label_smoothing must be in [0, 1], got {label_smoothing}")
    if process_group is not None and shard == "rows":
        if vocab_offset is not None or vocab_size is not None:
            raise ValueError("vocab_offset / vocab_size apply to shard='vocab' only")
        return _RowShardedCrossEntropy.apply(logits, target, reduction, ignore_index,
                                             label_smoothing, process_group)
    if shard not in ("vocab", "rows"):
        raise ValueError(f"shard must be 'vocab' or 'rows', got {shard!r}")
    if process_group is not None:
        import torch.distributed as dist
        off, V = shard_layout(dist.get_rank(process_group), dist.get_world_size(process_group),
                              logits.shape[1], vocab_offset, vocab_size)
        return _ShardedCrossEntropy.apply(logits, target, reduction, ignore_index,
                                          label_smoothing, process_group, off, V)
    return _FusedCrossEntropy.apply(logits, target, reduction, ignore_index, label_smoothing)


def cross_entropy_loss(
    logits: torch.Tensor,
    target: torch.Tensor,
    weight=None,
    reduction: str = "mean",
    ignore_index: int = -100,
    label_smoothing: float = 0.0,
) -> torch.Tensor:
    """Drop-in for F.cross_entropy (fused_cross_entropy.py:360-380).

    As in the reference, a class `weight` is not fused: that case is handed to
    torch's own cross_entropy.
    """
    if weight is not None:
        return torch.nn.functional.cross_entropy(
            logits, target, weight=weight, reduction=reduction,
            ignore_index=ignore_index, label_smoothing=label_smoothing)
    return fused_cross_entropy(logits, target, reduction=reduction,
                               ignore_index=ignore_index, label_smoothing=label_smoothing)
