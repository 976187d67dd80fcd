"""Host logic of the pipelined engine loop (TickEngine.tick_pipelined / flush), no GPU: the tick launch is replaced by
a fake device that runs each planned tick at once, in launch order, the way the stream would -- every seat's slot
counts the frames it has produced since its last bind and emits a stop code at a chosen frame -- so the same request
stream can be driven through tick() and tick_pipelined() and their deliveries compared: the same frames per request
in the same order, the same stop reasons and frame counts, the speculative frame of a stopped seat dropped, slots of
seats whose budget runs out refilled in the same tick as in the synchronous loop, and no slot released twice."""
import numpy as np
import pytest

from fake_engine import fake_engine


def drive(pipelined, n_seats=4, n_req=30, calls=80, seed=0):
    rng = np.random.default_rng(seed)
    budgets = rng.integers(3, 12, n_req)
    stop_at = {r: int(rng.integers(1, 8)) for r in range(n_req) if rng.random() < 0.4}
    eng, dev, released = fake_engine(n_seats, lambda s, k: stop_at.get(s.rid) == k)
    for r in range(n_req):
        eng.submit(np.arange(int(rng.integers(1, 4))), int(budgets[r]), rid=r, seed=r + 1)
    out = {}
    step = eng.tick_pipelined if pipelined else eng.tick
    for _ in range(calls):
        for s, code, cb0, pcm in step():
            out.setdefault(s.rid, []).append((code, cb0, None if pcm is None else tuple(pcm.tolist())))
    if pipelined:
        for s, code, cb0, pcm in eng.flush():
            out.setdefault(s.rid, []).append((code, cb0, None if pcm is None else tuple(pcm.tolist())))
    return eng, dev, released, out, stop_at, budgets


@pytest.mark.parametrize("seed", [0, 1, 2, 3])
def test_pipelined_deliveries_equal_the_synchronous_ones(seed):
    se, sdev, srel, sync, stop_at, budgets = drive(False, seed=seed)
    pe, pdev, prel, pipe, _, _ = drive(True, seed=seed)
    assert sync == pipe
    assert not se.pending and not pe.pending and not se.active and not pe.active
    # one release per request in both loops (which slot a request gets may differ: releases are ordered differently)
    assert len(srel) == len(prel) == len(sync) and not pe._early
    assert sorted(se.free) == sorted(pe.free) == list(range(4))
    for rid, rows in sync.items():
        frames = sum(p is not None for _, _, p in rows)
        if rid in stop_at and stop_at[rid] < budgets[rid]:
            assert rows[-1][0] == 1 and rows[-1][2] is None and frames == stop_at[rid]
        else:
            assert frames == budgets[rid] and all(c == 0 for c, _, _ in rows)
        # a request's frames come from its own slot's consecutive device frames
        assert [cb0 for _, cb0, _ in rows] == list(range(len(rows)))
    assert pe.stats["frames"] == se.stats["frames"] == sum(sum(p is not None for *_, p in v) for v in sync.values())
    assert pe.stats["completed"] == se.stats["completed"] == len(sync)
    # the pipelined loop ran one speculative frame per sampler stop that was not the seat's last budgeted frame
    spec = sum(1 for r in sync if r in stop_at and stop_at[r] + 1 < budgets[r])
    assert sum(pdev.ticks) == sum(sdev.ticks) + spec


def test_synchronous_tick_refuses_while_a_pipelined_tick_is_in_flight():
    eng, _, _, _, _, _ = drive(True, calls=0)
    eng.tick_pipelined()
    with pytest.raises(RuntimeError):
        eng.tick()
    eng.flush()
    eng.tick()


def test_codec_budget_only_for_pipelined_ticks():
    """A pipelined tick's codec part runs beside the next tick's main part, so it is launched within the codec's SM
    budget; a synchronous tick's codec part runs alone and keeps every SM."""
    eng, dev, _ = fake_engine(4)
    for i in range(3):
        eng.submit(np.arange(3) + i, 10)
    eng.tick()
    eng.tick()
    eng.tick_pipelined()
    eng.tick_pipelined()
    eng.flush()
    eng.tick()
    assert dev.beside == [False, False, True, True, False]
