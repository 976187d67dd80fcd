"""A TickEngine whose device is replaced by a host model, for tests of the host logic with no GPU: the real
TickEngine bookkeeping (admission, planning, delivery, pipelining, cancel) runs unchanged, and each planned tick is
"run" at once, in launch order as the stream would run it.  Every slot counts the frames it has produced since its
last bind; a seat's sampler emits a stop code at the frame `stop(seat, k)` names; its PCM at frame k is
PCM_COLS int64 words of pcm_value(seat, k)."""
import time
import types

import numpy as np

from maya2_native_b200.engine import TickConfig, TickEngine, Voice

PCM_COLS = 4


def pcm_value(seat, k):
    return int(np.asarray(seat.prompt).sum()) * 31 + k


def pcm_bytes(seat_prompt, k):
    return np.full(PCM_COLS, int(np.asarray(seat_prompt).sum()) * 31 + k, np.int64).tobytes()


class FakeDevice:
    def __init__(self, eng, stop, delay=0.0):
        self.eng = eng
        self.delay = delay                    # seconds each launched tick takes (a slow device)
        self.stop = stop                      # (seat, device frame index) -> True when the sampler stops there
        self.count = {}                       # slot -> frames produced since the slot's last bind
        self.owner = {}                       # slot -> id of the seat bound there
        self.ticks = []                       # the seat count of every launched tick
        self.beside = []                      # per launched tick: its codec part runs beside the next tick's main part

    def bind(self, s):
        self.eng._claim(s)
        self.count[s.slot] = 0
        self.owner[s.slot] = id(s)

    def launch(self, dec, new, beside=True):
        eng = self.eng
        tp = eng.make_plan(dec, new)
        seats = dec + new
        self.ticks.append(len(seats))
        self.beside.append(beside)
        if self.delay:
            time.sleep(self.delay)
        hv = np.zeros((len(seats), 2 + PCM_COLS), np.int64)
        for i, s in enumerate(seats):
            assert self.owner[s.slot] == id(s), "a tick ran a seat on a slot that was rebound under it"
            k = self.count[s.slot]
            self.count[s.slot] = k + 1
            hv[i, 0] = 1 if self.stop(s, k) else 0
            hv[i, 1] = k
            hv[i, 2:] = pcm_value(s, k)
        eng.commit(tp)
        return tp, types.SimpleNamespace(numpy=lambda: hv), types.SimpleNamespace(synchronize=lambda: None)


def fake_engine(n_seats, stop=lambda s, k: False, capacity=2048, max_inline_rows=16, delay=0.0):
    """(engine, fake device, list of released slots)."""
    eng = TickEngine.__new__(TickEngine)
    eng.cfg = TickConfig(max_seats=n_seats, capacity=capacity, max_inline_rows=max_inline_rows, min_frames=0)
    eng.device = None
    eng.guards = None
    eng.stats = {"ticks": 0, "admitted": 0, "completed": 0, "frames": 0, "prefill_rows": 0, "eager_prefill_rows": 0}
    eng.active, eng.pending = [], []
    eng.free = list(range(n_seats))[::-1]
    eng._early, eng._inflight, eng._readout, eng._custom = set(), None, None, set()
    eng.buckets = tuple(b for b in (1, 2, 4, 8, 16, 32) if b < n_seats) + (n_seats,)
    eng.max_rows = eng.buckets[-1] + max_inline_rows
    eng.row_buckets = tuple(b for b in (1, 2, 4, 8, 16, 32, 64, 128) if b < eng.max_rows) + (eng.max_rows,)
    eng.ctx_buckets = (capacity,)
    released = []

    def free(slot):
        released.append(slot)
        eng.backbone.lengths_cpu[slot] = 0

    eng.backbone = types.SimpleNamespace(lengths_cpu=[0] * (n_seats + 1), free=free)
    dev = FakeDevice(eng, stop, delay)
    eng._bind = dev.bind
    eng._launch_tick = dev.launch
    eng.prepare_voice = lambda ids: Voice(np.asarray(ids, np.int64), None, len(ids))
    eng._ids = iter(range(10 ** 6))
    eng._rng = np.random.default_rng(0)
    return eng, dev, released
