"""Multi-GPU column-parallel linear on 2 real GPUs (NCCL, one process per GPU): the
fused epilogue all-gather (P2P stores into CUDA IPC peer buffers) and the NCCL
all-gather path must both give the unsharded result bit for bit on every rank, also
over repeated calls where rank 0 reads each result late (a device-side delay before
its copy) while rank 1 runs its next call, whose stores land in rank 0's buffers.
Skipped where the machine has a single GPU."""
from __future__ import annotations

import os
import socket
from datetime import timedelta

import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu


def _port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank(rank, world, port, q):
    import torch.distributed as dist

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world,
                            timeout=timedelta(seconds=60), device_id=dev)
    try:
        import fp8linear_b200 as f
        from fp8linear_b200 import sharding as S
        from fp8linear_b200.capi import CApi

        M, K, N = 1000, 1024, 1536
        g = torch.Generator(device="cpu").manual_seed(0)
        x = torch.randn(M, K, generator=g).bfloat16().to(dev)
        w = (torch.randn(N, K, generator=g) * 0.02).bfloat16().to(dev)
        b = (torch.randn(N, generator=g) * 0.02).bfloat16().to(dev)
        wq, ws = f.quantize_weight(w)
        wqs, wss, bs = S.shard_columns(wq, ws, b, world, rank)
        capi = CApi()
        fused = S.FusedColumnParallel(M, N, torch.bfloat16, dev, peer=capi)
        xs = [(x * (1.0 + 0.25 * j)).bfloat16() for j in range(5)]
        fulls = [f.fp8_linear(xj, wq, ws, b) for xj in xs]
        nccl_ok = [bool(torch.equal(S.column_parallel_linear(xj, wqs, wss, bs, f.fp8_linear,
                                                              world), full))
                   for xj, full in zip(xs[:2], fulls[:2])]
        # No collective between rank 0's late read of call j and rank 1's call j + 1:
        # rank 1's next stores reach rank 0's buffers while rank 0's stream still waits.
        fused_ok = []
        for xj, full in zip(xs, fulls):
            out = fused(xj, wqs, wss, bs, capi)
            if rank == 0:
                torch.cuda._sleep(20_000_000)  # ~10 ms on the device before the read
            fused_ok.append(bool(torch.equal(out.clone(), full)))
        torch.cuda.synchronize(dev)
        fused.close()
        q.put((rank, all(nccl_ok), all(fused_ok)))
    except Exception as e:  # report and leave the group
        q.put((rank, "error", repr(e)[:300]))
    finally:
        dist.barrier()
        dist.destroy_process_group()


def test_column_parallel_two_gpus():
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    procs = [ctx.Process(target=_rank, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=180)
    alive = [p for p in procs if p.is_alive()]
    for p in alive:
        p.kill()
    assert not alive
    res = [q.get(timeout=5) for _ in range(2)]
    assert all(r[1:] == (True, True) for r in res), res
