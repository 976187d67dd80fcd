"""Multi-rank host logic on CPU (gloo, world size 2): the replicas' reduction used by bench.py -- the timed
durations take the max over ranks and the delivered frames the sum (every rank is an independent replica; there is
no collective on the decode path)."""
import os
import socket

import pytest
import torch.multiprocessing as mp


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, out):
    import datetime

    import torch.distributed as dist

    import bench
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    try:
        dev_ms = 100.0 + 10 * rank        # rank 1 is the slower replica
        e2e_ms = 150.0 - 20 * rank        # rank 0 is slower end to end
        frames = 1000 + rank
        e2e_frames = 2000 + 3 * rank
        out[rank] = bench.reduce_over_ranks(dev_ms, e2e_ms, frames, e2e_frames, world, "cpu")
        dist.barrier()
    finally:
        dist.destroy_process_group()


def test_reduce_over_ranks_gloo():
    world = 2
    port = _free_port()
    with mp.Manager() as m:
        out = m.dict()
        mp.spawn(_worker, args=(world, port, out), nprocs=world, join=True)
        res = dict(out)
    expect = (110.0, 150.0, 2001.0, 4003.0)
    for r in range(world):
        assert res[r] == pytest.approx(expect), res


def test_reduce_over_ranks_single():
    import bench
    assert bench.reduce_over_ranks(1.0, 2.0, 3, 4, 1, "cpu") == (1.0, 2.0, 3, 4)
