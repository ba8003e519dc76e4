"""Multi-rank sharding logic on CPU ranks (gloo, world size 2 and 4), with the oracle
port as each rank's linear: sharded results must equal the unsharded result bit for
bit. A rank that fails makes the others' collective end with an error, not a hang.

The fused all-gather's host logic (handle exchange, column offsets, the two buffers
used in turn, the ordering all-reduce, collective release) runs here with a stand-in
for the peer buffers: files mapped shared into every rank, written by a host-side
"kernel" that stores this rank's block into every rank's buffer."""
from __future__ import annotations

import ctypes
import os
import socket
import time
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


class ShmPeer:
    """Stand-in for the C ABI's peer buffers and fused op on CPU ranks: a buffer is a
    file under ``root`` mapped shared (torch.from_file) into every rank that opens it;
    its "handle" is the file name. ``fp8_linear_allgather`` computes this rank's block
    with the oracle and writes it into every output pointer, row by row."""

    def __init__(self, root: str):
        self.root = root
        self.maps: dict[int, tuple[torch.Tensor, str | None]] = {}
        self.n = 0

    def peer_alloc(self, nbytes):
        path = os.path.join(self.root, f"buf_{os.getpid()}_{self.n}")
        self.n += 1
        t = torch.from_file(path, shared=True, size=nbytes, dtype=torch.uint8)
        t.zero_()
        self.maps[t.data_ptr()] = (t, path)
        return t.data_ptr(), path.encode().ljust(64, b"\0")

    def peer_open(self, handle):
        path = handle.rstrip(b"\0").decode()
        t = torch.from_file(path, shared=True, size=os.path.getsize(path), dtype=torch.uint8)
        self.maps[t.data_ptr()] = (t, None)
        return t.data_ptr()

    def peer_close(self, ptr):
        self.maps.pop(ptr)

    def peer_free(self, ptr):
        _, path = self.maps.pop(ptr)
        os.unlink(path)

    def peer_tensor(self, ptr, nbytes, device):
        return self.maps[ptr][0]

    def fp8_linear_allgather(self, x, wq, ws, bias, out_ptrs, ldo, workspace=None):
        blk = oracle_linear(x, wq, ws, bias).bfloat16().contiguous()
        M, n = blk.shape
        for p in out_ptrs:
            for m in range(M):
                ctypes.memmove(p + m * ldo * 2, blk[m].data_ptr(), n * 2)


def _fused_worker(rank, world, port, root, single_buffer, q):
    """Four calls with different activations; rank 0 reads each result only after a
    delay, while the other ranks go on to their next call (which stores into rank 0's
    buffers). Every read must still see that call's own result."""
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=30))
    try:
        from fp8linear_b200 import sharding as S

        x0, wq, ws, b = _inputs(M=32, K=64, N=48)
        wqs, wss, bs = S.shard_columns(wq, ws, b, world, rank)
        fused = S.FusedColumnParallel(32, 48, torch.bfloat16, torch.device("cpu"),
                                      peer=ShmPeer(root))
        if single_buffer:  # the unsafe form: every call writes the same buffer
            fused.out_ptrs = lambda buf, f=fused, o=S.FusedColumnParallel.out_ptrs: o(f, 0)
            fused.views = [fused.views[0], fused.views[0]]
        same = []
        for j in range(4):
            x = (x0 * (j + 1)).bfloat16()
            out = fused(x, wqs, wss, bs)
            if rank == 0:
                time.sleep(0.3)
            got = out.clone()
            same.append(bool(torch.equal(got, oracle_linear(x, wq, ws, b).bfloat16())))
        fused.close()
        q.put((rank, "ok", tuple(same)))
    except Exception as e:
        q.put((rank, "error", type(e).__name__ + ": " + str(e)[:200]))
    finally:
        dist.destroy_process_group()


def _run_fused(world, root, single_buffer=False):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_fused_worker, args=(r, world, port, root, single_buffer, q))
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


@pytest.mark.parametrize("world", [2, 3])
def test_fused_column_parallel_buffers_in_turn(world, tmp_path):
    """Every result read (rank 0 reading late) equals the unsharded result, and every
    buffer file is freed by close()."""
    res = _run_fused(world, str(tmp_path))
    assert len(res) == world
    assert all(v == ("ok", (True,) * 4) for v in res.values()), res
    assert not any(tmp_path.iterdir())


def test_fused_single_buffer_hazard_is_detected(tmp_path):
    """The same test on the unsafe one-buffer form sees rank 0's late reads overwritten
    by the other rank's next call: the check above is sensitive to the hazard."""
    res = _run_fused(2, str(tmp_path), single_buffer=True)
    assert res[0][0] == "ok" and not all(res[0][1]), res
