"""Host logic of the pipelined engine loop (TickEngine.tick_pipelined / flush), no GPU: the tick launch is replaced by
a fake device that runs each planned tick at once, in launch order, the way the stream would -- every seat's slot
counts the frames it has produced since its last bind and emits a stop code at a chosen frame -- so the same request
stream can be driven through tick() and tick_pipelined() and their deliveries compared: the same frames per request
in the same order, the same stop reasons and frame counts, the speculative frame of a stopped seat dropped, slots of
seats whose budget runs out refilled in the same tick as in the synchronous loop, and no slot released twice."""
import types

import numpy as np
import pytest

from maya2_native_b200.engine import TickConfig, TickEngine

PCM_COLS = 4


class FakeDevice:
    def __init__(self, eng, stop_at):
        self.eng = eng
        self.stop_at = stop_at                  # rid -> device frame index at which the sampler emits a stop code
        self.count = {}                         # slot -> frames produced since the slot's last bind
        self.owner = {}                         # slot -> rid bound there
        self.ticks = []                         # the seat count of every launched tick

    def bind(self, s):
        self.eng._claim(s)
        self.count[s.slot] = 0
        self.owner[s.slot] = s.rid

    def launch(self, dec, new):
        eng = self.eng
        tp = eng.make_plan(dec, new)
        seats = dec + new
        self.ticks.append(len(seats))
        hv = np.zeros((len(seats), 2 + PCM_COLS), np.int64)
        for i, s in enumerate(seats):
            assert self.owner[s.slot] == s.rid, "a tick ran a seat on a slot that was rebound under it"
            k = self.count[s.slot]
            self.count[s.slot] = k + 1
            hv[i, 0] = 1 if self.stop_at.get(s.rid) == k else 0
            hv[i, 1] = s.rid * 1000 + k
            hv[i, 2:] = s.rid * 7919 + k
        eng.commit(tp)
        return tp, types.SimpleNamespace(numpy=lambda: hv), types.SimpleNamespace(synchronize=lambda: None)


def fake_engine(n_seats, stop_at):
    eng = TickEngine.__new__(TickEngine)
    eng.cfg = TickConfig(max_seats=n_seats, capacity=256, max_inline_rows=16, min_frames=0)
    eng.guards = None
    eng.stats = {"ticks": 0, "admitted": 0, "completed": 0, "frames": 0, "prefill_rows": 0, "eager_prefill_rows": 0}
    eng.active, eng.pending = [], []
    eng.free = list(range(n_seats))[::-1]
    eng._early, eng._inflight, eng._readout = set(), None, None
    eng.buckets = (1, 2, 4, 8)
    eng.row_buckets = (1, 2, 4, 8, 16, 32)
    eng.max_rows = 32
    eng.ctx_buckets = (256,)
    released = []

    def free(slot):
        released.append(slot)
        eng.backbone.lengths_cpu[slot] = 0

    eng.backbone = types.SimpleNamespace(lengths_cpu=[0] * (n_seats + 1), free=free)
    dev = FakeDevice(eng, stop_at)
    eng._bind = dev.bind
    eng._launch_tick = dev.launch
    eng._ids = iter(range(10 ** 6))
    eng._rng = np.random.default_rng(0)
    return eng, dev, released


def drive(pipelined, n_seats=4, n_req=30, calls=80, seed=0):
    rng = np.random.default_rng(seed)
    budgets = rng.integers(3, 12, n_req)
    stop_at = {r: int(rng.integers(1, 8)) for r in range(n_req) if rng.random() < 0.4}
    eng, dev, released = fake_engine(n_seats, stop_at)
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
        assert [cb0 % 1000 for _, cb0, _ in rows] == list(range(len(rows)))
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
