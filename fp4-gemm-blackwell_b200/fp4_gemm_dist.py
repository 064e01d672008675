"""Multi-GPU NVFP4 linear layers on one node (one process per GPU).

The reference runs on one device (SURVEY: no collective anywhere).  Two ways
to spread the cached linear over the GPUs of a node, both built on the
single-GPU kernels of ``fp4_gemm``:

* ``DataParallelFP4Linear`` -- rows of the activations are independent, so
  every rank holds the whole weight cache and runs its own rows; no
  collective.  ``row_range`` splits a global batch into 128-row-aligned parts.
* ``ColumnParallelFP4Linear`` -- the weight is N-sharded: rank p quantizes
  and keeps only its 128-row slice of W (the same bytes as that slice of the
  full cache, because quantization is row-local and scale atoms cover 128
  rows).  Each rank computes its output columns, then one NCCL all-gather of
  equal-size, zero-padded slices and a re-layout assemble [M, N] on every
  rank.

Host logic (shard plans, gather and re-layout) is separated from the GPU
kernels so it can be tested with ``gloo`` process groups on CPU.
"""
from __future__ import annotations

from dataclasses import dataclass

import torch
import torch.distributed as dist

TILE = 128  # rows per scale atom; shards start on these boundaries


@dataclass(frozen=True)
class ColumnShard:
    """Output columns [start, stop) owned by one rank; `width` is the padded gather width."""
    start: int
    stop: int
    width: int

    @property
    def cols(self) -> int:
        return self.stop - self.start


def plan_column_shards(n: int, world: int) -> list[ColumnShard]:
    """Split N output features into `world` contiguous 128-row-aligned shards.

    Tiles of 128 rows are dealt out as evenly as possible (the first ranks get
    one more tile when they do not divide evenly); a rank may own none when
    there are fewer tiles than ranks.  Every shard is gathered at the width of
    the largest one."""
    if n <= 0 or world <= 0:
        raise ValueError("n and world must be positive")
    tiles = (n + TILE - 1) // TILE
    base, extra = divmod(tiles, world)
    counts = [base + (1 if p < extra else 0) for p in range(world)]
    width = max(counts) * TILE
    shards, t = [], 0
    for c in counts:
        start = min(t * TILE, n)
        stop = min((t + c) * TILE, n)
        shards.append(ColumnShard(start, stop, width))
        t += c
    return shards


def row_range(m: int, world: int, rank: int, align: int = TILE) -> tuple[int, int]:
    """Rows [start, stop) of an M-row batch for `rank` in a data-parallel split (align-row chunks)."""
    chunks = (m + align - 1) // align
    base, extra = divmod(chunks, world)
    first = rank * base + min(rank, extra)
    count = base + (1 if rank < extra else 0)
    return min(first * align, m), min((first + count) * align, m)


def gather_columns(local: torch.Tensor, shards: list[ColumnShard], group=None) -> torch.Tensor:
    """All-gather per-rank column slices [M, cols_p] into the full [M, N] on every rank.

    Each slice is zero-padded to the common width, gathered with one
    ``all_gather_into_tensor`` into [P*M, width] (rank-major), then re-laid out."""
    world = dist.get_world_size(group)
    rank = dist.get_rank(group)
    assert len(shards) == world
    m = local.shape[0]
    width = shards[0].width
    assert local.shape[1] == shards[rank].cols, (local.shape, shards[rank])
    send = torch.zeros(m, width, dtype=local.dtype, device=local.device)
    send[:, : local.shape[1]] = local
    recv = torch.empty(world * m, width, dtype=local.dtype, device=local.device)
    dist.all_gather_into_tensor(recv, send, group=group)
    recv = recv.view(world, m, width)
    return torch.cat([recv[p, :, : shards[p].cols] for p in range(world)], dim=1)


class DataParallelFP4Linear:
    """Replicated weight cache; each rank runs the rows it owns (no collective)."""

    def __init__(self, weight: torch.Tensor, bias: torch.Tensor = None):
        import fp4_gemm
        self.cache = fp4_gemm.FP4WeightCache(weight, bias)

    def forward(self, x_local: torch.Tensor, sync: bool = False) -> torch.Tensor:
        return self.cache.forward(x_local, sync=sync)

    def free(self):
        self.cache.free()


class ColumnParallelFP4Linear:
    """N-sharded weight cache with an all-gather of the output columns.

    `weight` is the full [N, K] BF16 weight (each rank slices its own rows);
    the output of ``forward`` is the full [M, N] on every rank."""

    def __init__(self, weight: torch.Tensor, bias: torch.Tensor = None, group=None):
        import fp4_gemm
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        self.n, self.k = weight.shape
        self.shards = plan_column_shards(self.n, self.world)
        sh = self.shards[self.rank]
        self.cache = None
        if sh.cols > 0:
            b = bias[sh.start:sh.stop] if bias is not None else None
            self.cache = fp4_gemm.FP4WeightCache(weight[sh.start:sh.stop], b)

    def local_forward(self, x: torch.Tensor) -> torch.Tensor:
        sh = self.shards[self.rank]
        if self.cache is None:
            return torch.empty(x.reshape(-1, self.k).shape[0], 0, dtype=torch.bfloat16, device=x.device)
        return self.cache.forward(x.reshape(-1, self.k), sync=False)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        lead = x.shape[:-1]
        out = gather_columns(self.local_forward(x), self.shards, self.group)
        return out.reshape(*lead, self.n)

    def free(self):
        if self.cache is not None:
            self.cache.free()
