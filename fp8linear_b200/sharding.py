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

    Every rank owns an [M, N_total] output buffer in symmetric memory (mapped into every
    other rank's address space). ``__call__`` runs the fused op on this rank's channel
    block: each output box is stored to this GPU's buffer and, with P2P stores over
    NVLink, to every peer's buffer at this rank's column offset; a one-element NCCL
    all-reduce then orders every rank's writes before anyone reads the result. No
    separate all-gather or interleave copy runs.
    """

    def __init__(self, M: int, N_total: int, dtype: torch.dtype, device: torch.device,
                 group=None):
        import torch.distributed._symmetric_memory as symm

        self.group = group if group is not None else dist.group.WORLD
        self.world = dist.get_world_size(self.group)
        self.rank = dist.get_rank(self.group)
        self.M, self.N_total = M, N_total
        column_range(N_total, self.world, self.rank)  # validates the split
        self.buf = symm.empty(M, N_total, dtype=dtype, device=device)
        self.hdl = symm.rendezvous(self.buf, self.group)
        offset = self.buf.data_ptr() - self.hdl.buffer_ptrs[self.rank]
        self.bases = [int(b) + offset for b in self.hdl.buffer_ptrs]
        self.flag = torch.zeros(1, device=device)

    def out_ptrs(self) -> list[int]:
        """This rank's first output column in every rank's buffer, own buffer first."""
        n_local = self.N_total // self.world
        col = self.rank * n_local * self.buf.element_size()
        order = [self.rank] + [r for r in range(self.world) if r != self.rank]
        return [self.bases[r] + col for r in order]

    def __call__(self, x, wq_shard, ws_shard, bias_shard, capi, workspace=None):
        capi.fp8_linear_allgather(x, wq_shard, ws_shard, bias_shard, self.out_ptrs(),
                                  ldo=self.N_total, workspace=workspace)
        if self.world > 1:
            dist.all_reduce(self.flag, group=self.group)
        return self.buf
