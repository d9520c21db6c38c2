"""Host-side logic of the multi-GPU benchmark path, on two gloo ranks (CPU):
the job time is the slowest rank's and the job rate counts every rank's units."""
import os
import socket

import pytest
import torch.distributed as dist
import torch.multiprocessing as mp


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    import datetime
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60))
    import bench
    ms = [3.0, 5.0][rank]
    job = bench.max_over_ranks(ms, world)
    rate = bench.job_rate(1000.0, world, job)
    q.put((rank, job, rate))
    dist.barrier()
    dist.destroy_process_group()


def test_two_rank_timing_reduction():
    world, port = 2, _free_port()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    res = sorted(q.get(timeout=10) for _ in range(world))
    for rank, job, rate in res:
        assert job == 5.0                     # slowest rank
        assert rate == pytest.approx(1000.0 * 2 / 5e-3)


def test_single_rank_is_identity():
    import bench
    assert bench.max_over_ranks(7.5, 1) == 7.5
    assert bench.job_rate(10.0, 1, 2.0) == pytest.approx(5000.0)
