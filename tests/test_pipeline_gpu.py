"""The pipelined engine loop (TickEngine.tick_pipelined: tick t+1 launched before tick t is read) against the
synchronous one (TickEngine.tick, the reference's loop of maya3/engine.py:514-630): per request the same frames --
stop code, cb0 and PCM bit for bit -- the same stop reasons and frame counts, including a seat its sampler stops
(whose speculative frame in the next tick is dropped) and seats whose budget runs out (released and refilled in the
tick that follows, as in the synchronous loop).

Every tick of both runs has the same seat count (the queue never runs dry and the speculative seat fills the tick its
replacement waits), and every linear layer at this size runs at the same M in both, so per-row results do not
depend on which other seats share a tick and the streams must be identical."""
import numpy as np
import pytest
import torch

from maya2_native_b200 import weights as WG
from maya2_native_b200.config import TINY
from maya2_native_b200.engine import TickConfig, TickEngine

pytestmark = pytest.mark.gpu

CALLS = 48


def run(W, cuda, pipelined):
    cfg = TickConfig(max_seats=2, capacity=64, max_inline_rows=8)
    eng = TickEngine(TINY, W, cfg, device=cuda)
    rng = np.random.default_rng(5)
    reqs = []

    def submit(n):
        for _ in range(n):
            i = len(reqs)
            reqs.append(eng.submit(rng.integers(0, TINY.backbone.vocab, 3), 40 if i == 0 else 6 + i % 5,
                                   rid=i, seed=100 + i))

    submit(5)
    streams = {}
    step = eng.tick_pipelined if pipelined else eng.tick
    for call in range(CALLS):
        out = step()
        for s, code, cb0, pcm in out:
            streams.setdefault(s.rid, []).append((code, cb0, None if pcm is None else pcm.tobytes()))
        if call == 0:
            with torch.inference_mode():     # request 0 stops on its sampler as soon as its minimum frames are out
                eng.cb0.aeos_bias[reqs[0].slot] = 1e4
            if pipelined:
                with pytest.raises(RuntimeError):
                    eng.tick()
        if len(eng.pending) < 3:
            submit(3)
    if pipelined:
        for s, code, cb0, pcm in eng.flush():
            streams.setdefault(s.rid, []).append((code, cb0, None if pcm is None else pcm.tobytes()))
    status = eng.device_status()
    stats = dict(eng.stats)
    eng.close()
    return reqs, streams, stats, status


def test_pipelined_loop_delivers_the_synchronous_streams(cuda):
    W = {k: v.to(cuda) for k, v in WG.generate(WG.all_shapes(TINY), seed=3).items()}
    sreqs, sync, sstats, st1 = run(W, cuda, False)
    preqs, pipe, pstats, st2 = run(W, cuda, True)
    assert st1 == 0 and st2 == 0
    assert sreqs[0].stop in ("aeos", "aeos_argmax", "aeos_tau", "aeos_hazard"), sreqs[0].stop
    assert preqs[0].stop == sreqs[0].stop
    done = [r.rid for r in sreqs if r.stop is not None and preqs[r.rid].stop is not None]
    assert len(done) >= 8, done
    for rid in done:
        a, b = sreqs[rid], preqs[rid]
        assert (a.stop, a.frames) == (b.stop, b.frames), rid
        assert sync[rid] == pipe[rid], rid
        assert sum(p is not None for _, _, p in pipe[rid]) == b.frames
    # the sampler-stopped request's last row carries its stop code and no PCM in both loops
    assert sync[0][-1][0] != 0 and sync[0][-1][2] is None and pipe[0][-1] == sync[0][-1]
    # the pipelined run delivered every frame it counted (the dropped speculative frame is not one of them)
    assert pstats["frames"] == sum(sum(p is not None for _, _, p in v) for v in pipe.values())


def stream_of(eng, seat, step):
    out = []
    while seat.stop is None:
        for s, code, cb0, pcm in step():
            if s is seat:
                out.append((code, cb0, None if pcm is None else pcm.tobytes()))
    return out


def test_cancel_with_a_tick_in_flight_hands_a_clean_slot_to_the_next_request(cuda):
    """cancel() of a decoding request while its next tick is in flight (TickEngine.cancel): the slot is released at
    once and the request admitted into it next decodes exactly as on a fresh engine -- the slot's reset is
    stream-ordered behind the speculative tick that still wrote to it."""
    W = {k: v.to(cuda) for k, v in WG.generate(WG.all_shapes(TINY), seed=9).items()}
    cfg = TickConfig(max_seats=1, capacity=64, max_inline_rows=8, stops=False)
    rng = np.random.default_rng(2)
    pa, pb = rng.integers(0, TINY.backbone.vocab, 5), rng.integers(0, TINY.backbone.vocab, 4)
    ref = TickEngine(TINY, W, cfg, device=cuda)
    want = stream_of(ref, ref.submit(pb, 8, sampling={"seed": 5}), ref.tick)
    ref.close()
    eng = TickEngine(TINY, W, cfg, device=cuda)
    a = eng.submit(pa, 40, sampling={"seed": 4})
    for _ in range(4):
        eng.tick_pipelined()
    assert eng.cancel(a) and a.stop == "cancelled" and not eng.cancel(a)
    b = eng.submit(pb, 8, sampling={"seed": 5})
    got = stream_of(eng, b, eng.tick_pipelined)
    eng.flush()
    assert got == want
    assert eng.stats["cancelled"] == 1 and eng.device_status() == 0
    eng.close()
