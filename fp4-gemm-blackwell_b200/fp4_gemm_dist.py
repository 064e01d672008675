"""Multi-GPU NVFP4 linear layers on one node (one process per GPU).

The reference runs on one device (it has no collective anywhere).  Two ways
to spread the cached linear over the GPUs of a node, both built on the
single-GPU kernels of ``fp4_gemm``:

* ``DataParallelFP4Linear`` -- rows of the activations are independent, so
  every rank holds the whole weight cache and runs its own rows; no
  collective.  ``row_range`` splits a global batch into 128-row-aligned parts.
* ``ColumnParallelFP4Linear`` -- the weight is N-sharded: rank p quantizes
  and keeps only its 128-row slice of W (the same bytes as that slice of the
  full cache, because quantization is row-local and scale atoms cover 128
  rows).  Each rank computes its output columns and the result is assembled
  as [M, N] on every rank in one of these modes:
    - "epilogue": every rank's [M, N] buffer is mapped by every other rank
      (CUDA IPC), and the GEMM epilogue stores every output piece into all
      ranks' buffers (TMA bulk stores of 16 x 64 pieces: 128-byte rows, which
      SM stores over NVLink need for full rate), so the transfer overlaps
      the GEMM tile by tile; a flag barrier on the GPU (``PeerFlagBarrier``:
      one warp signals every peer and waits for every peer's signal) then
      orders the ranks.  No gather buffer, no re-layout, no collective.
      Needs N a multiple of 8.
    - "p2p": the same mapped buffers, but the GEMM writes only this rank's
      buffer, in row chunks, and a side stream pushes each finished chunk to
      every peer with a strided copy-engine copy while the next chunk is
      computed; then the flag barrier.  Any M.
    - "auto" (the default): "epilogue" where it applies (N a multiple of 8),
      else "p2p".
    - "nccl": one NCCL all-gather of equal-size, zero-padded slices and a
      re-layout.

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


class PeerFlagBarrier:
    """The column-parallel ranks' ordering step without a collective.

    Every rank owns a zeroed array of 8 uint64 flag slots, mapped by every
    other rank with CUDA IPC.  ``wait()`` queues fp4b_peer_barrier on the
    current stream: it stores the next epoch into this rank's slot of every
    peer's array and waits (on the GPU, bounded) until every peer has stored
    that epoch into this rank's array.  Every rank of the group must call
    ``wait()`` the same number of times, in the same order (the epochs then
    agree).  One barrier serves all the linears of a group (``for_group``).
    If a peer does not arrive within 10 s the wait gives up and records code
    10 in the device error word (``fp4_gemm.device_error()``)."""

    _by_group: dict = {}

    def __init__(self, group, device):
        import fp4_gemm
        self.group = group
        self.device = device
        self.rank = dist.get_rank(group)
        self.world = dist.get_world_size(group)
        self.flags = torch.zeros(8, dtype=torch.int64, device=device)
        mine = fp4_gemm.ipc_handle(self.flags)
        everyone = [None] * self.world
        dist.all_gather_object(everyone, mine, group=group)
        self.peer_ranks = [q for q in range(self.world) if q != self.rank]
        self._mapped = [(fp4_gemm.ipc_open(everyone[q][0], everyone[q][1], device), everyone[q][1])
                        for q in self.peer_ranks]
        self.epoch = 0

    @classmethod
    def for_group(cls, group, device) -> "PeerFlagBarrier":
        """The group's barrier, created on first use (a collective call: every rank at once)."""
        key = (id(group), str(device))
        b = cls._by_group.get(key)
        if b is None:
            b = cls._by_group[key] = cls(group, device)
        return b

    def wait(self):
        import fp4_gemm
        self.epoch += 1
        fp4_gemm.peer_barrier(self.flags, [p for p, _ in self._mapped], self.peer_ranks, self.rank, self.epoch)

    def close(self):
        """Unmap the peers' arrays (after the device has drained) and forget the barrier."""
        import fp4_gemm
        torch.cuda.synchronize(self.device)
        for ptr, off in self._mapped:
            fp4_gemm.ipc_close(ptr, off, self.device)
        self._mapped = []
        dist.barrier(group=self.group)  # no peer still maps this rank's array
        PeerFlagBarrier._by_group.pop((id(self.group), str(self.device)), None)

    @classmethod
    def close_all(cls):
        """Close every barrier of this process (before destroy_process_group)."""
        for b in list(cls._by_group.values()):
            b.close()


def peer_targets(peer_bases: dict, rank: int, world: int, buf: int, cap: int, n: int, start: int) -> list:
    """Device addresses where this rank's first output column lands in every other
    rank's double buffer [2, cap, n] (BF16): buffer `buf`, row 0, column `start`."""
    return [peer_bases[q] + 2 * (buf * cap * n + start) for q in range(world) if q != rank]


_COPY_STREAMS = {}  # device -> side stream of the p2p mode's peer copies


def row_chunks(m: int, min_rows: int = 1024, max_chunks: int = 4) -> list:
    """Row ranges [r0, r1) of the p2p mode's GEMM chunks: at most max_chunks,
    each at least min_rows (a multiple of 128) except the last."""
    size = max(min_rows, -(-m // max_chunks))
    size = -(-size // TILE) * TILE
    return [(r0, min(m, r0 + size)) for r0 in range(0, m, size)]


class ColumnParallelFP4Linear:
    """N-sharded weight cache; the output columns of all ranks are assembled.

    `weight` is the full [N, K] BF16 weight (each rank slices its own rows);
    the output of ``forward`` is the full [M, N] on every rank.  In the
    mapped-buffer modes ("auto", "epilogue", "p2p") it is a view of one of
    two per-layer buffers that the ranks write into each other: work queued
    before this rank's next ``forward`` of the layer may read it (the peers
    write the same buffer again in the forward after that, once this rank
    has passed the next one's barrier)."""

    def __init__(self, weight: torch.Tensor, bias: torch.Tensor = None, group=None, mode: str = "auto"):
        import fp4_gemm
        if mode not in ("auto", "p2p", "epilogue", "nccl"):
            raise ValueError("mode must be 'auto', 'p2p', 'epilogue' or 'nccl'")
        self.group = group
        self.mode = mode
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        self.n, self.k = weight.shape
        self.device = weight.device
        self.shards = plan_column_shards(self.n, self.world)
        sh = self.shards[self.rank]
        self.cache = None
        if sh.cols > 0:
            b = bias[sh.start:sh.stop] if bias is not None else None
            self.cache = fp4_gemm.FP4WeightCache(weight[sh.start:sh.stop], b)
        self._bias_ok = bias is None or bias.dtype == torch.bfloat16  # p2p fuses a BF16 bias
        self._bufs = None       # [2, cap, N] BF16, written by every rank
        self._peer_bases = {}   # rank -> (address of its _bufs in this process, IPC offset)
        self._flip = 0
        self._barrier = None

    def uses_p2p(self, m: int) -> bool:
        """Whether a forward of M rows assembles through the mapped buffers ("p2p"
        or "epilogue"); the same answer on every rank for the same M (the ranks
        must agree)."""
        if self.mode == "nccl" or self.world == 1 or self.device.type != "cuda" or not self._bias_ok or m <= 0:
            return False
        if self.mode == "epilogue":
            return self.n % 8 == 0
        return True

    def _epilogue(self, m: int) -> bool:
        """Whether a mapped-buffer forward of M rows has the GEMM epilogue store the
        peers' copies ("epilogue", and "auto" where the rows are 16-byte aligned)
        rather than the copy engine ("p2p")."""
        return self.mode == "epilogue" or (self.mode == "auto" and self.n % 8 == 0)

    def _ensure_buffers(self, m: int):
        import fp4_gemm
        if self._bufs is not None and self._bufs.shape[1] >= m:
            return
        if self._bufs is not None:
            # The host runs ahead of the GPU: this rank's previous GEMM may still be
            # storing through the peer mappings.  Its stream, which also holds the
            # previous call's rank-ordering step (after which every peer's stores
            # into this rank's old buffer are done), must drain before anything is
            # unmapped or freed.
            torch.cuda.synchronize(self.device)
        self._close_peers()
        cap = ((m + 127) // 128) * 128
        self._bufs = torch.empty(2, cap, self.n, dtype=torch.bfloat16, device=self.device)
        self._barrier = PeerFlagBarrier.for_group(self.group, self.device)
        mine = fp4_gemm.ipc_handle(self._bufs)
        everyone = [None] * self.world
        dist.all_gather_object(everyone, (mine[0], mine[1], cap), group=self.group)
        assert all(e[2] == cap for e in everyone), "ranks disagree on the batch size"
        for q, (h, off, _) in enumerate(everyone):
            if q != self.rank:
                self._peer_bases[q] = (fp4_gemm.ipc_open(h, off, self.device), off)

    def _close_peers(self):
        import fp4_gemm
        for ptr, off in self._peer_bases.values():
            fp4_gemm.ipc_close(ptr, off, self.device)
        self._peer_bases = {}

    def local_forward(self, x: torch.Tensor) -> torch.Tensor:
        sh = self.shards[self.rank]
        if self.cache is None:
            return torch.empty(x.reshape(-1, self.k).shape[0], 0, dtype=torch.bfloat16, device=x.device)
        return self.cache.forward(x.reshape(-1, self.k), sync=False)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        lead = x.shape[:-1]
        x2 = x.reshape(-1, self.k)
        m = x2.shape[0]
        if not self.uses_p2p(m):
            out = gather_columns(self.local_forward(x2), self.shards, self.group)
            return out.reshape(*lead, self.n)
        import fp4_gemm
        self._ensure_buffers(m)
        self._flip ^= 1
        cap = self._bufs.shape[1]
        out = self._bufs[self._flip, :m]
        sh = self.shards[self.rank]
        bases = {q: b for q, (b, _) in self._peer_bases.items()}
        if self._epilogue(m):
            if sh.cols > 0:
                peers = peer_targets(bases, self.rank, self.world, self._flip, cap, self.n, sh.start)
                fp4_gemm.run_cached_peers(x2, self.cache, out[:, sh.start:sh.stop], peers)
            # Every rank's tiles are in every buffer once all ranks have passed this point.
            self._barrier.wait()
            return out.reshape(*lead, self.n)
        cur = torch.cuda.current_stream(self.device)
        side = _COPY_STREAMS.get(self.device)
        if side is None:
            side = _COPY_STREAMS[self.device] = torch.cuda.Stream(self.device)
        side.wait_stream(cur)
        if sh.cols > 0:
            pitch = 2 * self.n
            for r0, r1 in row_chunks(m):
                fp4_gemm.run_cached_into(x2[r0:r1], self.cache, out[r0:r1, sh.start:sh.stop])
                side.wait_stream(cur)
                src = out[r0, sh.start:].data_ptr()
                with torch.cuda.stream(side):
                    for dst in peer_targets(bases, self.rank, self.world, self._flip, cap, self.n, sh.start):
                        fp4_gemm.copy2d(dst + r0 * pitch, pitch, src, pitch, 2 * sh.cols, r1 - r0, self.device)
        with torch.cuda.stream(side):
            # After this rank's copies; every peer's columns are here once it completes.
            self._barrier.wait()
        cur.wait_stream(side)
        return out.reshape(*lead, self.n)

    def free(self):
        if self._bufs is not None:
            torch.cuda.synchronize(self.device)
            self._close_peers()
            dist.barrier(group=self.group)  # no rank still maps this rank's buffers
            self._bufs = None
        if self.cache is not None:
            self.cache.free()
