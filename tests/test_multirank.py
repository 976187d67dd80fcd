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


def _box_worker(rank, world, port, out):
    import datetime

    import torch.distributed as dist

    import bench
    from maya2_native_b200.router import poisson_arrivals, share
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    try:
        # every replica derives its own round-robin share of the same seeded arrival stream
        arr = poisson_arrivals(100.0, 3.0, seed=5)
        idx = share(len(arr), rank, world)
        got = [None] * world
        dist.all_gather_object(got, idx.tolist())
        ttfa = [10.0 + rank, 20.0 + rank] if rank == 0 else [30.0]
        local = (ttfa, 1000 * (rank + 1), 6.0 + rank, 230.0 - rank, rank, len(idx), 0)
        out[rank] = (len(arr), got, bench.summarize_box(local, world, 256, 2500.0))
        dist.barrier()
    finally:
        dist.destroy_process_group()


def test_box_router_shares_and_summary_gloo():
    """configs[4] across two replicas: the round-robin shares partition the arrival stream, and the box summary sums
    the frames over replicas, divides by the longest window and takes TTFA percentiles over all the window's
    arrivals (those still without audio at its end included, with their wait so far)."""
    world = 2
    port = _free_port()
    with mp.Manager() as m:
        out = m.dict()
        mp.spawn(_box_worker, args=(world, port, out), nprocs=world, join=True)
        res = dict(out)
    n, shares, summ = res[0]
    assert sorted(shares[0] + shares[1]) == list(range(n)) and not set(shares[0]) & set(shares[1])
    assert abs(len(shares[0]) - len(shares[1])) <= 1
    for r in range(world):
        assert res[r][2] == summ
    assert summ["audio_s_per_s"] == pytest.approx(3000 * 0.08 / 7.0, abs=0.05)
    assert summ["offered_audio_s_per_s"] == pytest.approx(0.9 * 2500.0 * 2)
    assert summ["window_arrivals"] == 3 and summ["arrivals"] == n and summ["without_audio_at_end"] == 1
    assert summ["ttfa_p50_ms"] == pytest.approx(20.0)
    assert summ["mean_busy_seats_per_gpu"] == pytest.approx(229.5)


def _dead_peer_worker(rank, world, port, out):
    import datetime
    import time

    import torch.distributed as dist

    import bench
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=3))
    if rank == 1:          # this replica fails between steps: it never joins the reduction
        out[rank] = "left"
        return
    t0 = time.perf_counter()
    try:
        bench.reduce_over_ranks(1.0, 2.0, 3, 4, world, "cpu")
        out[rank] = "no error"
    except RuntimeError as e:      # the process group's timeout ends the collective with an error
        out[rank] = ("error", time.perf_counter() - t0, type(e).__name__)


def test_reduction_fails_fast_when_a_replica_dies():
    """A replica that leaves between steps never joins the timing reduction; the surviving rank's collective ends
    with an error after the process group's timeout instead of waiting forever (no GPU involved)."""
    world = 2
    port = _free_port()
    with mp.Manager() as m:
        out = m.dict()
        ctx = mp.spawn(_dead_peer_worker, args=(world, port, out), nprocs=world, join=False)
        ctx.join(60)
        res = dict(out)
    assert res.get(1) == "left"
    assert isinstance(res.get(0), tuple) and res[0][0] == "error" and res[0][1] < 30, res
