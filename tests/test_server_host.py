"""The HTTP / WebSocket front (maya3/server.py:409-1060 behaviour) over replicas whose engines run the real TickEngine
host logic on a fake device (no GPU): the wire format of each endpoint, errors before audio, admission control
(max_pending, queue deadline), cancel on disconnect, voices, several contexts per socket, routing over two replicas
and a failed replica.  A request's first token id below 50 makes the fake sampler stop at that frame; frame k of a
request carries PCM words sum(prompt) * 31 + k."""
import asyncio
import base64
import json
import struct
import time

import numpy as np
import pytest

pytest.importorskip("aiohttp")
from aiohttp import WSMsgType
from aiohttp.test_utils import TestClient, TestServer

from fake_engine import fake_engine, pcm_bytes
from maya2_native_b200.server import Maya3Server, Replica, wav_header

VOCAB = 1000


def stop_rule(s, k):
    if int(s.prompt[0]) == 999:
        raise RuntimeError("device fault (test)")
    return int(s.prompt[0]) < 50 and k == int(s.prompt[0])


def build(n_rep=1, seats=4, delay=0.0, pipelined=False, **kw):
    reps = [Replica(fake_engine(seats, stop_rule, delay=delay)[0], name=f"r{i}", pipelined=pipelined)
            for i in range(n_rep)]
    return Maya3Server(reps, vocab=VOCAB, **kw)


def run(srv, fn):
    async def main():
        async with TestClient(TestServer(srv.app())) as client:
            return await fn(client)
    try:
        return asyncio.run(main())
    finally:
        srv.close()


def frames_of(prompt, n):
    return b"".join(pcm_bytes(prompt, k) for k in range(n))


@pytest.mark.parametrize("pipelined", [False, True])
def test_speech_streams_the_engine_frames(pipelined):
    srv = build(pipelined=pipelined)
    prompt = [60, 1, 2]

    async def go(c):
        r = await c.post("/v1/audio/speech", json={"input_ids": prompt, "max_frames": 5, "seed": 7})
        body = await r.read()
        return r.status, dict(r.headers), body
    status, headers, body = run(srv, go)
    assert status == 200, body
    assert headers["Content-Type"] == "audio/wav" and headers["X-Sample-Rate"] == "24000"
    assert headers["X-Encoding"] == "pcm_s16le" and headers["X-Maya3-Voice"] == "plain"
    assert body == wav_header() + frames_of(prompt, 5)
    riff, size = struct.unpack("<4sI", body[:8])
    assert riff == b"RIFF" and size == 0xFFFFFFFF


def test_speech_pcm_sse_and_sampler_stop():
    srv = build()

    async def go(c):
        r1 = await c.post("/v1/audio/speech", json={"input_ids": [3, 5], "max_frames": 20, "response_format": "pcm"})
        pcm = await r1.read()
        r2 = await c.post("/v1/audio/speech", json={"input_ids": [70], "max_frames": 4, "response_format": "pcm",
                                                    "stream_format": "sse"})
        events = [json.loads(line[6:]) for line in (await r2.text()).split("\n\n") if line.startswith("data: ")]
        return r1.status, pcm, r2.status, r2.headers["Content-Type"], events
    s1, pcm, s2, ctype, events = run(srv, go)
    assert s1 == 200 and pcm == frames_of([3, 5], 3)          # the sampler stopped at frame 3: three frames of audio
    assert s2 == 200 and ctype == "text/event-stream"
    assert events[-1] == {"type": "speech.audio.done", "usage": {"audio_s": 0.32, "frames": 4, "reason": "max_frames"}}
    audio = b"".join(base64.b64decode(e["audio"]) for e in events if e["type"] == "speech.audio.delta")
    assert audio == frames_of([70], 4)


def test_speech_errors_before_audio():
    srv = build()
    cases = [({"input": "hello"}, "input"), ({"input_ids": [1], "response_format": "mp3"}, "response_format"),
             ({"input_ids": [1], "speed": 2.0}, "speed"), ({"input_ids": [1], "seed": -1}, "seed"),
             ({"input_ids": [1], "temperature": 3}, "temperature"), ({"input_ids": [VOCAB]}, "input_ids"),
             ({"input_ids": [1], "max_frames": 0}, "max_frames"), ({"input_ids": [1], "language": "xx"}, "language"),
             ({"input_ids": [1], "voice": "nobody"}, "voice"), ({"input_ids": [1], "stream_format": "x"},
                                                               "stream_format")]

    async def go(c):
        out = []
        for body, _ in cases:
            r = await c.post("/v1/audio/speech", json=body)
            out.append((r.status, await r.json()))
        r = await c.post("/v1/audio/speech", data=b"not json", headers={"content-type": "application/json"})
        out.append((r.status, await r.json()))
        return out
    res = run(srv, go)
    for (body, param), (status, err) in zip(cases, res):
        assert status == 400, (body, err)
        assert err["error"]["code"] == "invalid_request" and err["error"]["param"] == param, (body, err)
        assert err["error"]["type"] == "invalid_request_error"
    assert res[-1][0] == 400
    assert "encoder" in res[1][1]["error"]["message"]


def test_text_requests_go_through_the_encode_hook():
    seen = []

    def encode(text, lang, voice):
        seen.append((text, lang, voice))
        return [60] + [ord(ch) % VOCAB for ch in text]
    srv = build(encode=encode)

    async def go(c):
        r = await c.post("/v1/audio/speech", json={"input": "  hello ", "max_frames": 2, "voice": "alloy"})
        return r.status, r.headers["X-Maya3-Language"], r.headers["X-Maya3-Voice"], await r.read()
    status, lang, voice, body = run(srv, go)
    assert status == 200 and lang == "en" and voice == "plain"
    assert seen == [("hello", "en", "plain")]
    assert body == wav_header() + frames_of([60] + [ord(ch) for ch in "hello"], 2)


def test_admission_control():
    """max_pending bounds the requests waiting for first audio; a request that gets none within the queue deadline
    is refused with 503 and cancelled in the engine (maya3/server.py:516-551)."""
    srv = build(seats=1, delay=0.01, queue_deadline_ms=300, max_pending=1)
    eng = srv.replicas[0].engine

    async def go(c):
        ws = await c.ws_connect("/v1/tts/stream")
        await ws.receive_json()                                            # metadata
        await ws.send_json({"type": "speak", "context_id": "long", "text_ids": [60], "max_frames": 1500})
        first = await ws.receive_json()                                    # the only seat is now taken
        r1 = await c.post("/v1/audio/speech", json={"input_ids": [61], "max_frames": 3})
        e1 = await r1.json()
        t0 = time.perf_counter()
        while eng.pending and time.perf_counter() - t0 < 2:                # the refused request left the queue
            await asyncio.sleep(0.01)
        left = len(eng.pending)
        srv.max_pending = 0
        r2 = await c.post("/v1/audio/speech", json={"input_ids": [61], "max_frames": 3})
        e2 = await r2.json()
        await ws.close()
        return first, r1.status, e1, left, r2.status, r2.headers.get("Retry-After"), e2
    first, s1, e1, left, s2, retry, e2 = run(srv, go)
    assert first["type"] == "audio"
    assert s1 == 503 and e1["error"]["code"] == "overloaded" and "deadline" in e1["error"]["message"]
    assert left == 0
    assert s2 == 503 and retry == "1" and "max_pending" in e2["error"]["message"]


def test_websocket_protocol():
    srv = build(ws_max_contexts=2, delay=0.002)

    async def go(c):
        ws = await c.ws_connect("/v1/tts/stream")
        meta = await ws.receive_json()
        await ws.send_json({"type": "ping"})
        pong = await ws.receive_json()
        await ws.send_json({"type": "speak", "context_id": "a", "text_ids": [60, 2], "max_frames": 3})
        await ws.send_json({"type": "speak", "context_id": "b", "text_ids": [61], "max_frames": 1500,
                            "binary": True})
        await ws.send_json({"type": "speak", "context_id": "c", "text_ids": [62], "max_frames": 3})
        await ws.send_json({"type": "speak", "context_id": "a", "text_ids": [62], "max_frames": 3})
        await ws.send_bytes(b"\x00")
        audio = {"a": b"", "b": b""}
        ends, errors, cancelled = {}, [], False
        while "b" not in ends:
            msg = await ws.receive()
            if msg.type == WSMsgType.BINARY:
                n = struct.unpack("<I", msg.data[:4])[0]
                cid = msg.data[4:4 + n].decode()
                audio[cid] += msg.data[4 + n:]
                if len(audio["b"]) >= 4 * len(pcm_bytes([61], 0)) and not cancelled:
                    await ws.send_json({"type": "cancel", "context_id": "b"})
                    cancelled = True
                continue
            m = json.loads(msg.data)
            if m["type"] == "audio":
                audio[m["context_id"]] += base64.b64decode(m["audio"])
            elif m["type"] == "end":
                ends[m["context_id"]] = m
            elif m["type"] == "error":
                errors.append(m)
        await ws.close()
        return meta, pong, audio, ends, errors
    meta, pong, audio, ends, errors = run(srv, go)
    assert meta == {"type": "metadata", "sample_rate": 24000, "encoding": "pcm_s16le", "channels": 1,
                    "max_contexts": 2, "languages": list(meta["languages"])}
    assert pong == {"type": "pong"}
    assert audio["a"] == frames_of([60, 2], 3)
    assert ends["a"]["reason"] == "max_frames" and ends["a"]["frames"] == 3 and ends["a"]["ttfa_ms"] is not None
    assert ends["b"]["reason"] == "cancelled"
    nb = len(audio["b"]) // len(pcm_bytes([61], 0))
    assert nb >= 4 and audio["b"] == frames_of([61], nb)
    codes = sorted(e["code"] for e in errors)
    assert codes == ["invalid_request", "invalid_request", "too_many_contexts"], errors


def test_closing_the_socket_cancels_its_requests():
    srv = build(delay=0.002)
    eng = srv.replicas[0].engine

    async def go(c):
        ws = await c.ws_connect("/v1/tts/stream")
        await ws.receive_json()
        await ws.send_json({"type": "speak", "context_id": "x", "text_ids": [60], "max_frames": 1500})
        while (await ws.receive_json())["type"] != "audio":
            pass
        busy = len(eng.active)
        await ws.close()
        t0 = time.perf_counter()
        while eng.active and time.perf_counter() - t0 < 2:
            await asyncio.sleep(0.01)
        return busy, len(eng.active), eng.stats.get("cancelled", 0)
    busy, after, cancelled = run(srv, go)
    assert busy == 1 and after == 0 and cancelled == 1


def test_voices():
    srv = build()
    eng = srv.replicas[0].engine

    async def go(c):
        r1 = await c.post("/v1/voices", json={"voice_id": "v1", "prefix_ids": [5, 6, 7]})
        b1 = await r1.json()
        r2 = await c.post("/v1/voices", json={"voice_id": "v1", "prefix_ids": [5]})
        lst = await (await c.get("/v1/voices")).json()
        r3 = await c.post("/v1/audio/speech", json={"input_ids": [60], "voice": "V1", "max_frames": 2})
        await r3.read()
        r4 = await c.delete("/v1/voices/v1")
        r5 = await c.post("/v1/audio/speech", json={"input_ids": [60], "voice": "v1"})
        r6 = await c.post("/v1/voices", json={"voice_id": "bad id", "prefix_ids": [5]})
        return r1.status, b1, r2.status, lst, r3.status, r3.headers["X-Maya3-Voice"], r4.status, r5.status, r6.status
    s1, b1, s2, lst, s3, voice, s4, s5, s6 = run(srv, go)
    assert s1 == 201 and b1["id"] == "v1" and b1["prefix_tokens"] == 3
    assert s2 == 409
    assert [v["id"] for v in lst["voices"]] == ["plain", "v1"]
    assert s3 == 200 and voice == "v1"
    assert s4 == 200 and s5 == 400 and s6 == 400


def test_health_models_and_routing_over_two_replicas():
    srv = build(n_rep=2, delay=0.002)

    async def go(c):
        h = await c.get("/health")
        hb = await h.json()
        m = await (await c.get("/v1/models")).json()
        rs = await asyncio.gather(*[c.post("/v1/audio/speech", json={"input_ids": [60 + i], "max_frames": 6})
                                    for i in range(6)])
        bodies = [await r.read() for r in rs]
        return h.status, hb, m, [r.status for r in rs], bodies
    hs, hb, m, statuses, bodies = run(srv, go)
    assert hs == 200 and hb["ready"] and len(hb["replicas"]) == 2
    assert m["data"][0]["id"] == "maya3"
    assert statuses == [200] * 6
    assert all(b == wav_header() + frames_of([60 + i], 6) for i, b in enumerate(bodies))
    assert all(r.stats["submitted"] >= 2 for r in srv.replicas)


def test_a_failed_replica_ends_its_requests_with_an_error():
    srv = build()

    async def go(c):
        r1 = await c.post("/v1/audio/speech", json={"input_ids": [999], "max_frames": 3})
        e1 = await r1.json()
        t0 = time.perf_counter()
        while srv.replicas[0].failed is None and time.perf_counter() - t0 < 2:
            await asyncio.sleep(0.01)
        h = await c.get("/health")
        r2 = await c.post("/v1/audio/speech", json={"input_ids": [60], "max_frames": 3})
        return r1.status, e1, h.status, (await h.json())["replicas"][0]["failed"], r2.status, await r2.json()
    s1, e1, hs, failed, s2, e2 = run(srv, go)
    assert s1 == 503 and e1["error"]["code"] == "internal"
    assert hs == 503 and "device fault" in failed
    assert s2 == 503 and e2["error"]["code"] == "unavailable"
