"""Sharded fused_cross_entropy kernels, two ranks on one GPU (gloo collectives).

The vocabulary-sharded path (fo_ce_shard_stats / fo_ce_shard_combine /
fo_ce_shard_bwd) and the row-sharded path (fo_ce_count_valid / fo_ce_rows_fwd
/ fo_ce_bwd) run as two spawned processes that share cuda:0 and exchange their
row statistics through a gloo process group.  None of these kernels waits on
another rank (every exchange is a host-side collective between launches), so
two processes on one GPU are safe, and the kernels' parity is checked on a box
with a single GPU.  Each rank's loss and gradient block must equal the oracle
on the whole matrix: fp32 rtol 1e-5, bf16/fp16 rtol 2e-2 (the standards of
test_fused_cross_entropy.py).  tests/test_multigpu.py runs the same paths over
NCCL when two GPUs are present.
"""
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


# (B, V, dtype, split): split None = equal blocks, else the first block's extent
CASES = [(64, 4096, torch.float32, None), (33, 5000, torch.float32, 1234),
         (256, 32000, torch.bfloat16, None), (17, 999, torch.float16, 7)]


def _worker(rank, port, q):
    import torch.distributed as dist
    from operators.fused_cross_entropy import fused_cross_entropy
    try:
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
        torch.cuda.set_device(0)
        dev = torch.device("cuda", 0)
        dist.init_process_group("gloo", rank=rank, world_size=WORLD)
        fails = []
        for ci, (B, V, dtype, split) in enumerate(CASES):
            g = torch.Generator().manual_seed(200 + ci)
            logits = (torch.randn(B, V, generator=g) * 3).to(dtype)
            target = torch.randint(0, V, (B,), generator=g)
            target[::6] = -100
            for red in ("none", "mean", "sum"):
                for ls in (0.0, 0.1):
                    rl, rg = oracle.fused_cross_entropy_grad(logits.float(), target,
                                                             reduction=red, label_smoothing=ls)
                    # vocabulary blocks
                    if split is None:
                        lo, hi = rank * V // WORLD, (rank + 1) * V // WORLD
                    else:
                        lo, hi = (0, split) if rank == 0 else (split, V)
                    x = logits[:, lo:hi].contiguous().to(dev).requires_grad_(True)
                    loss = fused_cross_entropy(x, target.to(dev), reduction=red,
                                               label_smoothing=ls, process_group=dist.group.WORLD,
                                               vocab_offset=lo, vocab_size=V)
                    loss.backward(torch.ones_like(loss))
                    if not (_close(loss.detach().cpu(), rl.to(dtype), dtype)
                            and _close(x.grad.cpu(), rg[:, lo:hi].to(dtype), dtype)):
                        fails.append(("vocab", B, V, str(dtype), red, ls))
                    # row blocks
                    if split is None:
                        r0, r1 = rank * B // WORLD, (rank + 1) * B // WORLD
                    else:
                        r0, r1 = (0, min(split, B)) if rank == 0 else (min(split, B), B)
                    x = logits[r0:r1].contiguous().to(dev).requires_grad_(True)
                    loss = fused_cross_entropy(x, target[r0:r1].to(dev), reduction=red,
                                               label_smoothing=ls, process_group=dist.group.WORLD,
                                               shard="rows")
                    loss.backward(torch.ones_like(loss))
                    want = rl[r0:r1] if red == "none" else rl
                    if not (_close(loss.detach().cpu(), want.to(dtype), dtype)
                            and _close(x.grad.cpu(), rg[r0:r1].to(dtype), dtype)):
                        fails.append(("rows", B, V, str(dtype), red, ls))
        dist.barrier()
        dist.destroy_process_group()
        q.put((rank, fails))
    except Exception as e:  # report instead of leaving the parent waiting
        q.put((rank, repr(e)))


def test_sharded_cross_entropy_two_ranks_one_gpu():
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
        for p in procs:
            p.join(timeout=60)
        for p in procs:
            if p.is_alive():
                p.terminate()
                p.join(timeout=10)
    for rank, res in out:
        assert isinstance(res, list), f"rank {rank}: {res}"
        assert not res, f"rank {rank} mismatches: {res}"
