"""Multi-rank sharding logic on CPU ranks (gloo, world size 2 and 4), with the oracle
port as each rank's linear: sharded results must equal the unsharded result bit for
bit. A rank that fails makes the others' collective end with an error, not a hang."""
from __future__ import annotations

import os
import socket
from datetime import timedelta

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from fp8linear_b200.sharding import column_range, row_range


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def oracle_linear(x, wq, ws, bias):
    """CPU restatement of fp8_linear on torch tensors (bf16 x, uint8 codes)."""
    from oracle import oracle as O

    x16 = x.contiguous().view(torch.int16).numpy().view(np.uint16)
    out = O.port_linear(x16, wq.numpy(), ws.numpy(), None, acc_dtype="float64",
                        round_out=False)
    out = torch.from_numpy(out)
    if bias is not None:
        out = out + bias.float()[None, :]
    return out


def _inputs(M=96, K=64, N=48, seed=0):
    from oracle import oracle as O

    g = torch.Generator().manual_seed(seed)
    x = torch.randn(M, K, generator=g).bfloat16()
    w = (torch.randn(N, K, generator=g) * 0.02).bfloat16()
    b = (torch.randn(N, generator=g) * 0.02).bfloat16()
    wq, ws = O.np_quantize_weight(w.view(torch.int16).numpy().view(np.uint16), O.BF16)
    return x, torch.from_numpy(wq), torch.from_numpy(ws), b


def _worker(rank, world, port, mode, fail_rank, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=20))
    try:
        from fp8linear_b200 import sharding as S

        x, wq, ws, b = _inputs()
        if mode == "rows":
            local = S.row_parallel_linear(x, wq, ws, b, oracle_linear, world, rank)
            parts = [None] * world
            dist.all_gather_object(parts, local)  # verification only
            got = torch.cat(parts)
        else:
            if rank == fail_rank:
                raise RuntimeError("injected failure before the all-gather")
            wqs, wss, bs = S.shard_columns(wq, ws, b, world, rank)
            got = S.column_parallel_linear(x, wqs, wss, bs, oracle_linear, world)
        full = oracle_linear(x, wq, ws, b)
        q.put((rank, "ok", bool(torch.equal(got, full))))
    except Exception as e:  # report, then leave the group
        q.put((rank, "error", type(e).__name__ + ": " + str(e)[:200]))
    finally:
        dist.destroy_process_group()


def _run(world, mode, fail_rank=-1):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, mode, fail_rank, q))
             for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
    alive = [p for p in procs if p.is_alive()]
    for p in alive:
        p.kill()
    assert not alive, "a rank hung"
    res = {}
    while not q.empty():
        r, status, payload = q.get()
        res[r] = (status, payload)
    return res


def test_row_range_partition():
    for M in (0, 1, 7, 4608, 18432):
        for world in (1, 2, 3, 4, 8):
            spans = [row_range(M, world, r) for r in range(world)]
            assert spans[0][0] == 0 and spans[-1][1] == M
            assert all(a[1] == b[0] for a, b in zip(spans, spans[1:]))
            sizes = [e - s for s, e in spans]
            assert max(sizes) - min(sizes) <= 1


def test_column_range():
    assert column_range(65536 * 0 + 3072, 8, 7) == (2688, 3072)
    with pytest.raises(ValueError):
        column_range(3072, 5, 0)
    with pytest.raises(ValueError):
        column_range(48, 4, 0)  # 12-column blocks break 16-byte rows


@pytest.mark.parametrize("world", [2, 4])
def test_row_sharded_equals_unsharded(world):
    res = _run(world, "rows")
    assert len(res) == world
    assert all(v == ("ok", True) for v in res.values()), res


@pytest.mark.parametrize("world", [2, 3])
def test_column_sharded_allgather_equals_unsharded(world):
    if 48 % world or (48 // world) % 8:
        world = 2
    res = _run(world, "cols")
    assert all(v == ("ok", True) for v in res.values()), res


def test_failed_rank_ends_collective_with_error():
    """Rank 1 raises before the all-gather: rank 0's collective ends with an error
    (gloo notices the peer leaving or the group timeout fires) instead of hanging."""
    res = _run(2, "cols", fail_rank=1)
    assert res[1][0] == "error" and "injected" in res[1][1]
    assert res[0][0] == "error"
