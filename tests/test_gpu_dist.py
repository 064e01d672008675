"""Multi-GPU cached linear on one node (NCCL): column-parallel N-shards with an
all-gather, and the data-parallel row split, against the single-GPU result.
Runs as child processes on 2 GPUs; skipped on a 1-GPU box."""
import os
import socket

import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, q):
    import datetime

    import torch.distributed as dist

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev,
                            timeout=datetime.timedelta(seconds=60))
    try:
        import fp4_gemm
        import fp4_gemm_dist as D
        from tests import workloads as W
        from tests.gpu_helpers import assert_gemm_close
        m, n, k = 512, 2880, 1024
        x, w, b = W.cached_linear_inputs(m, n, k, seed=3)
        xd, wd, bd = x.to(dev), w.to(dev), b.to(dev)
        tp = D.ColumnParallelFP4Linear(wd, bd)
        single = fp4_gemm.FP4WeightCache(wd, bd)
        # A small batch first, then the full one: the peer buffers grow while the
        # previous call's stores may still be in flight.
        assert torch.equal(tp.forward(xd[:256]), single.forward(xd[:256]))
        y = tp.forward(xd)
        ref = single.forward(xd)
        assert_gemm_close(y, ref.float(), f"column-parallel rank {rank}")
        # Column tiles of a shard run the same MMAs as in the full GEMM: every
        # assembly mode gives the single-GPU bytes exactly.
        assert tp.uses_p2p(m) and tp._epilogue(m)  # "auto": the epilogue stores to the peers
        assert torch.equal(y, ref), "column-parallel differs from one GPU"
        y2 = tp.forward(xd[:384])  # second buffer, fewer rows
        assert torch.equal(y2, single.forward(xd[:384]))
        assert torch.equal(tp.forward(xd), ref)  # first buffer again
        nc = D.ColumnParallelFP4Linear(wd, bd, mode="nccl")
        assert torch.equal(nc.forward(xd), ref)
        ep = D.ColumnParallelFP4Linear(wd, bd, mode="epilogue")  # the GEMM epilogue stores to the peers
        assert ep.uses_p2p(m)
        assert torch.equal(ep.forward(xd[:256]), single.forward(xd[:256]))
        assert torch.equal(ep.forward(xd), ref)
        assert torch.equal(ep.forward(xd[:100]), single.forward(xd[:100]))  # M <= 128: a pair's second CTA is padding
        ep.free()
        ce = D.ColumnParallelFP4Linear(wd, bd, mode="p2p")  # copy-engine pushes
        assert ce.uses_p2p(m) and not ce._epilogue(m)
        assert torch.equal(ce.forward(xd), ref)
        big = W.normal_bf16((2304, k), 1.0, 5).to(dev)  # several copy-engine row chunks (1024-row minimum)
        want_big = single.forward(big)
        assert torch.equal(ce.forward(big), want_big)
        assert torch.equal(tp.forward(big), want_big)  # auto: epilogue stores, several tiles per CTA pair
        small = tp.forward(xd[:100])  # auto at M <= 128: the epilogue stores too
        assert tp._epilogue(100)
        assert torch.equal(small, single.forward(xd[:100]))
        assert torch.equal(ce.forward(xd[:100]), small)  # copy-engine pushes of a single row chunk
        ce.free()
        nc.free()
        r0, r1 = D.row_range(m, world, rank)
        dp = D.DataParallelFP4Linear(wd, bd)
        yl = dp.forward(xd[r0:r1], sync=True)
        assert_gemm_close(yl, ref[r0:r1].float(), f"data-parallel rank {rank}")
        barrier = D.PeerFlagBarrier.for_group(None, dev)
        assert barrier.epoch >= 4  # one GPU flag barrier per p2p forward, no collective
        assert fp4_gemm.device_error() == 0
        tp.free()
        dp.free()
        single.free()
        D.PeerFlagBarrier.close_all()
        torch.cuda.synchronize()
        dist.barrier()
        q.put((rank, "ok"))
    except Exception as e:  # reported to the parent, which fails the test
        q.put((rank, repr(e)))
    finally:
        dist.destroy_process_group()


def test_column_and_data_parallel_two_gpus(cuda):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=300)
    codes = [p.exitcode for p in procs]
    for p in procs:
        if p.exitcode is None:
            p.kill()
    results = [q.get(timeout=10) for _ in procs] if all(c == 0 for c in codes) else []
    assert codes == [0, 0], f"rank exit codes {codes}"
    assert all(r == "ok" for _, r in results), results
