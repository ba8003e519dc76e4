"""Sharding of the FP8 linear across GPUs (one process per GPU, torch.distributed).

The path shards two natural ways; the reference has no multi-GPU code, so both are
new here.

* Token rows (M): rows are independent (per-token scales, per-row GEMM rows), so
  rank r takes a contiguous block of rows, the weight is replicated and no
  collective runs on the data path (``row_range`` / ``row_parallel_linear``).
* Output channels (N): rank r holds a contiguous block of weight rows with their
  per-channel scales and bias, computes ``out[:, block]`` for all tokens (every rank
  quantizes the full x, so the per-token scales are identical everywhere), and the
  blocks are all-gathered into ``[M, N]`` (``column_parallel_linear``). The
  all-gather delivers ``[P, M, N/P]``; one strided copy interleaves it into
  row-major ``[M, N]``.

Every function takes the per-rank linear as a callable so the same host logic runs
with the CUDA op on GPUs (NCCL) and with a CPU restatement in tests (gloo).
"""
from __future__ import annotations

from typing import Callable

import torch
import torch.distributed as dist

Linear = Callable[[torch.Tensor, torch.Tensor, torch.Tensor, torch.Tensor | None], torch.Tensor]


def row_range(M: int, world: int, rank: int) -> tuple[int, int]:
    """Contiguous block of rows of rank ``rank``; the first ``M % world`` ranks take one
    extra row."""
    if world <= 0 or not 0 <= rank < world:
        raise ValueError(f"bad rank {rank} of {world}")
    base, extra = divmod(M, world)
    start = rank * base + min(rank, extra)
    return start, start + base + (1 if rank < extra else 0)


def column_range(N: int, world: int, rank: int, align: int = 8) -> tuple[int, int]:
    """Equal contiguous block of output channels; each block must keep the kernel's
    16-byte output rows (``align`` bf16 columns)."""
    if N % world != 0 or (N // world) % align != 0:
        raise ValueError(f"N={N} does not split into {world} blocks of a multiple of {align}")
    n = N // world
    return rank * n, (rank + 1) * n


def row_parallel_linear(x: torch.Tensor, wq: torch.Tensor, ws: torch.Tensor,
                        bias: torch.Tensor | None, linear: Linear, world: int,
                        rank: int) -> torch.Tensor:
    """This rank's rows of ``linear(x)``; x is the full ``[M, K]`` batch (or already the
    local shard when ``world == 1``). No communication."""
    s, e = row_range(x.shape[0], world, rank)
    return linear(x[s:e], wq, ws, bias)


def shard_columns(wq: torch.Tensor, ws: torch.Tensor, bias: torch.Tensor | None, world: int,
                  rank: int):
    s, e = column_range(wq.shape[0], world, rank)
    return wq[s:e].contiguous(), ws[s:e].contiguous(), (
        None if bias is None else bias[s:e].contiguous())


def gather_columns(local: torch.Tensor, world: int, group=None) -> torch.Tensor:
    """All-gather ``[M, N/P]`` blocks from every rank into row-major ``[M, N]``."""
    M, n = local.shape
    local = local.contiguous()
    buf = torch.empty((world * M, n), dtype=local.dtype, device=local.device)
    dist.all_gather_into_tensor(buf, local, group=group)
    out = torch.empty((M, world * n), dtype=local.dtype, device=local.device)
    out.view(M, world, n).copy_(buf.view(world, M, n).permute(1, 0, 2))
    return out


def column_parallel_linear(x: torch.Tensor, wq_shard: torch.Tensor, ws_shard: torch.Tensor,
                           bias_shard: torch.Tensor | None, linear: Linear, world: int,
                           group=None) -> torch.Tensor:
    """``linear`` over this rank's channel block, then the all-gather to ``[M, N]``."""
    local = linear(x, wq_shard, ws_shard, bias_shard)
    if world == 1:
        return local
    return gather_columns(local, world, group)


class FusedColumnParallel:
    """N-shard linear with the all-gather fused into the GEMM epilogue.

    Every rank allocates two ``[M, N_total]`` output buffers as peer memory (plain CUDA
    IPC mappings over NVLink through the C ABI's ``fp8lin_peer_buffer_*``; no multicast
    object) and maps every other rank's two. Call j writes buffer ``j % 2``: the
    epilogue stores each output box to this GPU's buffer and, with P2P stores, to every
    peer's buffer at this rank's column offset; a one-element all-reduce on the stream
    then orders every rank's writes before anyone reads the result. No separate
    all-gather or interleave copy runs.

    Lifetime of a result: the tensor that call j returns is the buffer that call j + 2
    rewrites, on every rank. No rank starts call j + 2 before the all-reduce of call
    j + 1 has completed everywhere, and that all-reduce follows, on each rank's stream,
    everything the rank enqueued before making call j + 1. So a result stays intact for
    every read enqueued before the call after next; ``.clone()`` it to keep it longer.

    ``peer`` provides the buffer set-up (``peer_alloc``, ``peer_open``, ``peer_close``,
    ``peer_free``, ``peer_tensor``) and the fused op (``fp8_linear_allgather``); it
    defaults to the C ABI binding. ``close()`` releases the buffers collectively.
    """

    def __init__(self, M: int, N_total: int, dtype: torch.dtype, device: torch.device,
                 group=None, peer=None):
        self.group = group if group is not None else dist.group.WORLD
        self.world = dist.get_world_size(self.group)
        self.rank = dist.get_rank(self.group)
        self.M, self.N_total, self.dtype, self.device = M, N_total, dtype, torch.device(device)
        column_range(N_total, self.world, self.rank)  # validates the split
        if peer is None:
            from .capi import CApi

            peer = CApi()
        self.peer = peer
        self.elem = torch.empty((), dtype=dtype).element_size()
        self.nbytes = M * N_total * self.elem
        self.local: list[int] = []        # this rank's two buffers
        self.opened: list[int] = []       # peers' buffers mapped here
        self.bases: list[list[int]] = []  # per buffer: every rank's base address, by rank
        self.views: list[torch.Tensor] = []
        err = None
        try:
            for _ in range(2):
                ptr, handle = self.peer.peer_alloc(self.nbytes)
                self.local.append(ptr)
                handles = [None] * self.world
                dist.all_gather_object(handles, handle, group=self.group)
                bases = []
                for r in range(self.world):
                    if r == self.rank:
                        bases.append(ptr)
                    else:
                        q = self.peer.peer_open(handles[r])
                        self.opened.append(q)
                        bases.append(q)
                self.bases.append(bases)
                self.views.append(self.peer.peer_tensor(ptr, self.nbytes, self.device)
                                  .view(dtype).view(M, N_total))
        except Exception as e:  # every rank learns of a failed set-up before going on
            err = e
        ok = torch.tensor([0 if err is not None else 1], dtype=torch.int32,
                          device=self._coll_device())
        dist.all_reduce(ok, op=dist.ReduceOp.MIN, group=self.group)
        self.calls = 0
        self.closed = False
        self.flag = torch.zeros(1, device=self._coll_device())
        if int(ok.item()) != 1:
            self._release(collective=False)
            raise RuntimeError(f"peer buffer set-up failed on a rank: {err!r}")

    def _coll_device(self) -> torch.device:
        return torch.device("cpu") if dist.get_backend(self.group) == "gloo" else self.device

    def out_ptrs(self, buf: int) -> list[int]:
        """This rank's first output column in every rank's buffer ``buf``, own first."""
        n_local = self.N_total // self.world
        col = self.rank * n_local * self.elem
        order = [self.rank] + [r for r in range(self.world) if r != self.rank]
        return [self.bases[buf][r] + col for r in order]

    def __call__(self, x, wq_shard, ws_shard, bias_shard, capi=None, workspace=None):
        if self.closed:
            raise RuntimeError("FusedColumnParallel used after close()")
        buf = self.calls % 2
        self.calls += 1
        op = capi if capi is not None else self.peer
        op.fp8_linear_allgather(x, wq_shard, ws_shard, bias_shard, self.out_ptrs(buf),
                                ldo=self.N_total, workspace=workspace)
        if self.world > 1:
            dist.all_reduce(self.flag, group=self.group)
        return self.views[buf]

    def _release(self, collective: bool) -> None:
        self.views = []
        if collective:
            # every rank is done with the peers' buffers before any mapping goes away
            if self.device.type == "cuda":
                torch.cuda.synchronize(self.device)
            dist.barrier(group=self.group)
        for q in self.opened:
            self.peer.peer_close(q)
        self.opened = []
        if collective:
            dist.barrier(group=self.group)  # no rank maps this rank's buffers any more
        for p in self.local:
            self.peer.peer_free(p)
        self.local = []

    def close(self) -> None:
        """Unmap the peers' buffers and free this rank's (collective: every rank calls
        it, with none of the buffers' readers still in flight)."""
        if not self.closed:
            self.closed = True
            self._release(collective=True)

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()
