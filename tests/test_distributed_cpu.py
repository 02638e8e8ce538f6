"""Multi-process (world size 2, gloo, CPU) tests of the vocabulary-sharded
cross-entropy host logic: block layout, the all_gather of per-row statistics and
the combine rule reproduce the single-device loss.  The CUDA kernels of the same
path run in tests/test_multigpu.py on 2 GPUs."""
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

import oracle
from operators.fused_cross_entropy import shard_layout


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, V, uneven, q):
    try:
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
        dist.init_process_group("gloo", rank=rank, world_size=world)
        g = torch.Generator().manual_seed(5)
        B = 12
        logits = torch.randn(B, V, generator=g) * 2
        target = torch.randint(0, V, (B,), generator=g)
        target[3] = -100
        if uneven:
            bounds = [0, V // 3, V]
            off, Vfull = shard_layout(rank, world, bounds[rank + 1] - bounds[rank],
                                      vocab_offset=bounds[rank], vocab_size=V)
            block = logits[:, bounds[rank]:bounds[rank + 1]]
        else:
            vl = V // world
            off, Vfull = shard_layout(rank, world, vl)
            block = logits[:, off:off + vl]
        stats = oracle.ce_shard_stats(block, target, off).float()
        gathered = [torch.empty_like(stats) for _ in range(world)]
        dist.all_gather(gathered, stats)
        all_stats = torch.stack(gathered)
        res = {}
        for red in ("none", "mean", "sum"):
            for ls in (0.0, 0.1):
                got = oracle.ce_shard_combine(all_stats, target, Vfull, label_smoothing=ls,
                                              reduction=red)
                ref = oracle.fused_cross_entropy(logits.double(), target, reduction=red,
                                                 label_smoothing=ls)
                res[(red, ls)] = float((got - ref).abs().max())
        q.put((rank, res))
        dist.destroy_process_group()
    except Exception as e:  # report to the parent instead of hanging it
        q.put((rank, repr(e)))


@pytest.mark.parametrize("uneven", [False, True])
def test_vocab_sharded_ce_two_ranks_gloo(uneven):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, 1000, uneven, q)) for r in range(2)]
    for p in procs:
        p.start()
    out = [q.get(timeout=120) for _ in procs]
    for p in procs:
        p.join(timeout=60)
    for rank, res in out:
        assert isinstance(res, dict), f"rank {rank} failed: {res}"
        for k, err in res.items():
            assert err < 1e-4, (rank, k, err)


def _rows_worker(rank, world, port, bounds, q):
    try:
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
        dist.init_process_group("gloo", rank=rank, world_size=world)
        g = torch.Generator().manual_seed(9)
        B, V = bounds[-1], 777
        logits = torch.randn(B, V, generator=g) * 2
        target = torch.randint(0, V, (B,), generator=g)
        target[::5] = -100
        lo, hi = bounds[rank], bounds[rank + 1]
        res = {}
        for ls in (0.0, 0.1):
            part = oracle.ce_rows_partial(logits[lo:hi], target[lo:hi], label_smoothing=ls)
            parts = [torch.empty_like(part) for _ in range(world)]
            dist.all_gather(parts, part)
            for red in ("mean", "sum"):
                got = oracle.ce_rows_combine(torch.stack(parts), red)
                ref = oracle.fused_cross_entropy(logits.double(), target, reduction=red,
                                                 label_smoothing=ls)
                res[(red, ls)] = float((got - ref).abs())
        q.put((rank, res))
        dist.destroy_process_group()
    except Exception as e:  # report to the parent instead of hanging it
        q.put((rank, repr(e)))


@pytest.mark.parametrize("bounds", [[0, 20, 40], [0, 7, 40]])
def test_row_sharded_ce_two_ranks_gloo(bounds):
    """Row blocks (even and uneven): the per-rank (loss sum, valid rows) pairs
    summed over ranks give the single-device 'mean' and 'sum' losses."""
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rows_worker, args=(r, 2, port, bounds, q)) for r in range(2)]
    for p in procs:
        p.start()
    try:
        out = [q.get(timeout=120) for _ in procs]
    finally:
        for p in procs:
            p.join(timeout=60)
            if p.is_alive():
                p.terminate()
    for rank, res in out:
        assert isinstance(res, dict), f"rank {rank} failed: {res}"
        for k, err in res.items():
            assert err < 1e-9, (rank, k, err)


def test_shard_layout_rules():
    assert shard_layout(1, 4, 100) == (100, 400)
    assert shard_layout(0, 2, 30, vocab_offset=0, vocab_size=50) == (0, 50)
    with pytest.raises(ValueError):
        shard_layout(3, 4, 100, vocab_size=350)


def _peer_worker(rank, world, port, q):
    """Rank 1 fails to map rank 0's region (a simulated fo_peer_open error);
    rank 0 maps rank 1's.  Both must give up together and rank 0 must unmap
    what it mapped.  The library calls that would touch GPU memory are
    replaced by stand-ins (no pointer is ever dereferenced here)."""
    try:
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
        dist.init_process_group("gloo", rank=rank, world_size=world)
        from operators import _lib
        from operators import fused_cross_entropy as fce
        real_call, closed = _lib.call, []

        def fake_call(name, *args):
            if name == "fo_peer_export":
                args[2]._obj.value = 0  # byref(offset)
                return None
            if name == "fo_peer_open":
                if rank == 1:
                    raise RuntimeError("fo_peer_open: simulated mapping failure")
                args[2]._obj.value = 0x1000
                return None
            if name == "fo_peer_close":
                closed.append(args[1])
                return None
            return real_call(name, *args)

        _lib.call = fake_call
        try:
            fce._PeerRegions(dist.group.WORLD, torch.device("cpu"), 16)
            res = "no error"
        except fce._PeerUnavailable as e:
            res = ("unavailable", len(closed), str(e))
        dist.barrier()
        dist.destroy_process_group()
        q.put((rank, res))
    except Exception as e:  # report to the parent instead of hanging it
        q.put((rank, repr(e)))


def test_peer_regions_setup_failure_is_agreed():
    """The NVLink cross-entropy path is set up by every rank or by none: a
    mapping failure on one rank makes every rank fall back (no rank is left
    waiting on a peer that will never write)."""
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_peer_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    try:
        out = dict(q.get(timeout=120) for _ in procs)
    finally:
        for p in procs:
            p.join(timeout=60)
            if p.is_alive():
                p.terminate()
    assert isinstance(out[0], tuple) and out[0][0] == "unavailable", out
    assert isinstance(out[1], tuple) and out[1][0] == "unavailable", out
    assert out[0][1] == 1, f"rank 0 should unmap the one region it mapped: {out[0]}"
    assert out[1][1] == 0, out
