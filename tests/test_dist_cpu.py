"""Multi-GPU host logic on CPU: shard plans and the column all-gather with
2-rank gloo process groups (no GPU, no NCCL)."""
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

import fp4_gemm_dist as D


def test_plan_column_shards_cover_and_align():
    for n in (1, 127, 128, 129, 2880, 5120, 15360, 64):
        for world in (1, 2, 3, 4, 8):
            shards = D.plan_column_shards(n, world)
            assert len(shards) == world
            assert shards[0].start == 0 and shards[-1].stop == n
            for a, b in zip(shards, shards[1:]):
                assert a.stop == b.start
            for s in shards:
                assert s.cols == 0 or s.start % D.TILE == 0
                assert 0 <= s.cols <= s.width and s.width % D.TILE == 0
    s = D.plan_column_shards(2880, 8)  # 23 tiles over 8 ranks: 3,3,3,3,3,3,3,2
    assert [x.cols for x in s] == [384] * 7 + [192] and s[0].width == 384


def test_row_range_partitions_batch():
    for m in (1, 100, 2048, 8192, 1000):
        for world in (1, 2, 4, 8):
            parts = [D.row_range(m, world, r) for r in range(world)]
            assert parts[0][0] == 0 and parts[-1][1] == m
            for (a0, a1), (b0, b1) in zip(parts, parts[1:]):
                assert a1 == b0
            assert all(p0 % D.TILE == 0 or p0 == p1 for p0, p1 in parts)


def test_peer_targets_address_columns_in_peer_buffers():
    # bases of the peers' [2, cap, n] BF16 buffers; buffer 1, column 384
    bases = {0: 1 << 20, 2: 3 << 20, 3: 4 << 20}
    got = D.peer_targets(bases, rank=1, world=4, buf=1, cap=256, n=2880, start=384)
    step = 2 * (256 * 2880 + 384)
    assert got == [(1 << 20) + step, (3 << 20) + step, (4 << 20) + step]


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, n, m, k, q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        g = torch.Generator().manual_seed(0)
        x = torch.randn(m, k, generator=g)
        w = torch.randn(n, k, generator=g)
        shards = D.plan_column_shards(n, world)
        sh = shards[rank]
        # stand-in for the per-rank FP4 kernel: the exact product of the local rows
        local = x @ w[sh.start:sh.stop].t()
        full = D.gather_columns(local, shards)
        ok = torch.allclose(full, x @ w.t(), atol=1e-5)
        q.put((rank, bool(ok), tuple(full.shape)))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("n", [300, 2880])
def test_gather_columns_two_ranks_gloo(n):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, n, 37, 64, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
    codes = [p.exitcode for p in procs]
    for p in procs:
        if p.exitcode is None:
            p.kill()
    assert codes == [0, 0], f"rank exit codes {codes}"
    results = [q.get(timeout=10) for _ in procs]
    assert all(ok for _, ok, _ in results), results
    assert all(shape == (37, n) for _, _, shape in results)


def _leaving_worker(rank, world, port, q):
    import datetime
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=10))
    if rank == 1:
        os._exit(0)  # this rank leaves between steps, before its next collective
    shards = D.plan_column_shards(300, world)
    local = torch.zeros(5, shards[rank].cols)
    try:
        D.gather_columns(local, shards)
        q.put((rank, "returned"))
    except Exception as e:  # the survivor's collective ends with an error instead of waiting for good
        q.put((rank, type(e).__name__))
    # os._exit skips the queue's feeder thread: flush the message before leaving.
    q.close()
    q.join_thread()
    os._exit(0)


def test_rank_that_leaves_ends_the_survivors_collective_with_an_error():
    # Failure detection on the host: when one rank leaves, the other rank's
    # next collective (the column all-gather) raises within the process
    # group's short timeout rather than hanging.
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_leaving_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
    codes = [p.exitcode for p in procs]
    for p in procs:
        if p.exitcode is None:
            p.kill()
    assert codes == [0, 0], f"rank exit codes {codes}"
    rank, outcome = q.get(timeout=10)
    assert rank == 0 and outcome != "returned", outcome


def test_row_chunks_partition_rows():
    # The p2p mode's GEMM chunks: contiguous, cover [0, M), at most 4, 128-row
    # multiples of at least 1024 rows except the last.
    for m in (1, 100, 1024, 2048, 2304, 8192, 8200, 20000):
        ch = D.row_chunks(m)
        assert ch[0][0] == 0 and ch[-1][1] == m and len(ch) <= 4
        for (a0, a1), (b0, b1) in zip(ch, ch[1:]):
            assert a1 == b0 and (a1 - a0) % D.TILE == 0 and a1 - a0 >= 1024


def _layer_stub(mode, n, world=2, bias_ok=True):
    # The mode decisions of ColumnParallelFP4Linear are host logic; a stub
    # with just the fields they read stands in for a layer (which needs GPUs).
    lin = object.__new__(D.ColumnParallelFP4Linear)
    lin.mode, lin.n, lin.world, lin._bias_ok = mode, n, world, bias_ok
    lin.device = torch.device("cuda", 0)
    return lin


def test_column_parallel_mode_choice():
    auto = _layer_stub("auto", 2880)
    # auto: the GEMM epilogue stores to the peers where the output rows are
    # 16-byte aligned (N a multiple of 8), at any M; else copy-engine pushes.
    for m in (1, 128, 129, 8192):
        assert auto.uses_p2p(m) and auto._epilogue(m)
    odd = _layer_stub("auto", 2884 + 1)
    assert odd.uses_p2p(4096) and not odd._epilogue(4096)
    ce = _layer_stub("p2p", 2880)
    assert ce.uses_p2p(4096) and not ce._epilogue(4096)
    ep = _layer_stub("epilogue", 2880)
    assert ep.uses_p2p(4096) and ep._epilogue(4096) and ep.uses_p2p(1)
    assert not _layer_stub("epilogue", 2885).uses_p2p(4096)  # unaligned rows: the all-gather
    assert not _layer_stub("nccl", 2880).uses_p2p(4096)
    assert not _layer_stub("auto", 2880, world=1).uses_p2p(4096)
    assert not _layer_stub("auto", 2880, bias_ok=False).uses_p2p(4096)  # an fp32 bias is added after a gather
    with pytest.raises(ValueError):
        D.ColumnParallelFP4Linear(torch.zeros(128, 128), mode="ring")
