"""The HTTP / WebSocket front over a real engine replica on the GPU (its engine thread on the synchronous or the
pipelined loop): a request's PCM over HTTP (and over the WebSocket) is byte for byte what the same engine
configuration delivers to the same request driven directly
through TickEngine (seeded sampler streams, maya3/engine.py:430-433), with per-request cb0 sampling overrides --
temperature, top-k and top-p, the last of which switches the captured tick to its top-p form."""
import asyncio
import base64

import numpy as np
import pytest
import torch

pytest.importorskip("aiohttp")
from aiohttp.test_utils import TestClient, TestServer

from maya2_native_b200 import weights as WG
from maya2_native_b200.config import TINY
from maya2_native_b200.engine import TickConfig, TickEngine
from maya2_native_b200.server import Maya3Server, Replica

pytestmark = pytest.mark.gpu

REQS = [({"seed": 7}, 6), ({"seed": 11, "temperature": 0.5, "top_k": 10}, 5), ({"seed": 3, "top_p": 0.8}, 7)]


def engine(W, cuda):
    return TickEngine(TINY, W, TickConfig(max_seats=2, capacity=128, max_inline_rows=16), device=cuda)


def direct(W, cuda, ids, sampling, frames):
    eng = engine(W, cuda)
    s = eng.submit(ids, frames, sampling=sampling)
    pcm = b""
    while s.stop is None:
        for seat, _, _, p in eng.tick():
            if seat is s and p is not None:
                pcm += p.tobytes()
    eng.close()
    return pcm, s.stop


@pytest.mark.parametrize("pipelined", [False, True])
def test_server_streams_the_engine_pcm(cuda, pipelined):
    W = {k: v.to(cuda) for k, v in WG.generate(WG.all_shapes(TINY), seed=5).items()}
    ids = np.random.default_rng(1).integers(0, TINY.backbone.vocab, 9).tolist()
    want = [direct(W, cuda, ids, sp, n) for sp, n in REQS]
    srv = Maya3Server([Replica(engine(W, cuda), name="gpu0", pipelined=pipelined)], vocab=TINY.backbone.vocab)

    async def http(c, sp, n):
        r = await c.post("/v1/audio/speech", json={"input_ids": ids, "max_frames": n, "response_format": "pcm", **sp})
        return r.status, await r.read()

    async def go(c):
        # one request at a time, each alone as in the direct runs; the top-p request last, since the engine's top-p
        # switch stays on once a request has used it (maya3/engine.py:444-445)
        got = [await http(c, *REQS[0]), await http(c, *REQS[1])]
        ws = await c.ws_connect("/v1/tts/stream")
        await ws.receive_json()
        await ws.send_json({"type": "speak", "context_id": "c", "text_ids": ids, "max_frames": REQS[0][1],
                            **REQS[0][0]})
        audio, end = b"", None
        while end is None:
            m = await ws.receive_json()
            if m["type"] == "audio":
                audio += base64.b64decode(m["audio"])
            elif m["type"] in ("end", "error"):
                end = m
        await ws.close()
        got.append(await http(c, *REQS[2]))
        return got, audio, end

    async def main():
        async with TestClient(TestServer(srv.app())) as client:
            return await go(client)
    try:
        got, audio, end = asyncio.run(main())
    finally:
        status = srv.replicas[0].engine.device_status()
        srv.close()
    for (st, body), (pcm, stop) in zip(got, want):
        assert st == 200 and len(pcm) > 0
        assert body == pcm
    assert end["type"] == "end" and end["reason"] == want[0][1] and audio == want[0][0]
    assert status == 0
