"""Vocabulary- and row-sharded fused_cross_entropy on 2 GPUs (one process per GPU, NCCL).

Each rank holds a column block of the logits; the loss and this rank's block of
the gradient must equal the single-device result of the oracle on the whole
matrix (fp32 rtol 1e-5, bf16 rtol 2e-2 as in test_fused_cross_entropy.py).  The
vocabulary split runs twice: through the fused kernel that exchanges the row
statistics over NVLink peer memory (the default on one host), checked to have
been taken and to have had no timed-out wait, and with FLAGOPS_CE_P2P=0 through
the all-gather path.  Skipped when fewer than 2 GPUs are visible.  Ranks run as
spawned processes with a 60 s process-group timeout and NVLS off, and report
through a queue.
"""
import datetime
import os
import socket

import pytest
import torch

import oracle

pytestmark = pytest.mark.gpu
WORLD = 2


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _close(got, ref, dtype):
    if dtype == torch.float32:
        return bool(torch.allclose(got.float(), ref.float(), rtol=1e-5, atol=1e-6))
    scale = ref.float().abs().max().item()
    return bool(torch.allclose(got.float(), ref.float(), rtol=2e-2, atol=2e-5 * scale))


def _cases():
    # (B, V, dtype, split) — split None: equal blocks; else the first block's width
    # (the 1500-row case outgrows the peer regions' first 1024 rows; the 80000-
    # column case has rows past 64 KiB per rank, which the NVLink path runs with
    # a CTA per row instead of a warp)
    return [(64, 4096, torch.float32, None), (33, 5000, torch.float32, 1234),
            (256, 32000, torch.bfloat16, None), (17, 999, torch.float16, 500),
            (1500, 2048, torch.float32, None), (40, 80000, torch.float32, None)]


def _worker(rank, port, q):
    import torch.distributed as dist
    from operators.fused_cross_entropy import fused_cross_entropy
    try:
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
        torch.cuda.set_device(rank)
        dev = torch.device("cuda", rank)
        dist.init_process_group("nccl", rank=rank, world_size=WORLD,
                                timeout=datetime.timedelta(seconds=60), device_id=dev)
        fails = []
        for p2p in ("1", "0"):
            os.environ["FLAGOPS_CE_P2P"] = p2p
            fails += _run_cases(rank, dev, dist, fused_cross_entropy, rows=(p2p == "1"))
        import ctypes
        from operators import _lib
        from operators import fused_cross_entropy as fce
        if not isinstance(fce._PEER.get((id(dist.group.WORLD), rank)), fce._PeerRegions):
            fails.append("the NVLink peer-memory path was not taken")
        n = ctypes.c_uint(0)
        _lib.call("fo_ce_p2p_timeouts", ctypes.byref(n))
        if n.value:
            fails.append(f"{n.value} peer waits timed out")
        dist.barrier()
        dist.destroy_process_group()
        q.put((rank, fails))
    except Exception as e:  # report instead of leaving the parent waiting
        q.put((rank, repr(e)))


def _run_cases(rank, dev, dist, fused_cross_entropy, rows):
    fails = []
    for ci, (B, V, dtype, split) in enumerate(_cases()):
        g = torch.Generator().manual_seed(100 + ci)
        logits = (torch.randn(B, V, generator=g) * 3).to(dtype)
        target = torch.randint(0, V, (B,), generator=g)
        target[::7] = -100
        if split is None:
            lo, hi = rank * V // WORLD, (rank + 1) * V // WORLD
            kw = {} if V % WORLD == 0 else {"vocab_offset": lo, "vocab_size": V}
        else:
            lo, hi = (0, split) if rank == 0 else (split, V)
            kw = {"vocab_offset": lo, "vocab_size": V}
        for red in ("none", "mean", "sum"):
            for ls in (0.0, 0.1):
                x = logits[:, lo:hi].contiguous().to(dev).requires_grad_(True)
                loss = fused_cross_entropy(x, target.to(dev), reduction=red,
                                           label_smoothing=ls, process_group=dist.group.WORLD,
                                           **kw)
                loss.backward(torch.ones_like(loss))
                rl, rg = oracle.fused_cross_entropy_grad(logits.float(), target,
                                                         reduction=red, label_smoothing=ls)
                ok_l = _close(loss.detach().cpu(), rl.to(dtype), dtype)
                ok_g = _close(x.grad.cpu(), rg[:, lo:hi].to(dtype), dtype)
                if not (ok_l and ok_g):
                    fails.append((B, V, str(dtype), split, red, ls, ok_l, ok_g))
                if red == "mean" and ls == 0.0:
                    # forward only (no gradient slice written)
                    with torch.no_grad():
                        l2 = fused_cross_entropy(x.detach(), target.to(dev), reduction=red,
                                                 process_group=dist.group.WORLD, **kw)
                    if not _close(l2.cpu(), rl.to(dtype), dtype):
                        fails.append(("no-grad", B, V, str(dtype)))
                if not rows:
                    continue
                # the same batch split by rows instead
                r0, r1 = rank * B // WORLD, (rank + 1) * B // WORLD
                xr = logits[r0:r1].contiguous().to(dev).requires_grad_(True)
                lr = fused_cross_entropy(xr, target[r0:r1].to(dev), reduction=red,
                                         label_smoothing=ls, process_group=dist.group.WORLD,
                                         shard="rows")
                lr.backward(torch.ones_like(lr))
                want = rl[r0:r1] if red == "none" else rl
                if not (_close(lr.detach().cpu(), want.to(dtype), dtype)
                        and _close(xr.grad.cpu(), rg[r0:r1].to(dtype), dtype)):
                    fails.append(("rows", B, V, str(dtype), red, ls))
    return fails


@pytest.mark.skipif(torch.cuda.device_count() < WORLD, reason="needs 2 GPUs")
def test_vocab_sharded_cross_entropy_two_gpus():
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, port, q)) for r in range(WORLD)]
    for p in procs:
        p.start()
    try:
        out = [q.get(timeout=300) for _ in procs]
    finally:
        # never leave a rank holding a GPU: join, then end any rank still alive
        for p in procs:
            p.join(timeout=60)
        for p in procs:
            if p.is_alive():
                p.terminate()
                p.join(timeout=10)
    for rank, res in out:
        assert isinstance(res, list), f"rank {rank}: {res}"
        assert not res, f"rank {rank} mismatches: {res}"
