"""HTTP / WebSocket front over native engine replicas (maya3/server.py:409-1060 served by TickEngine).

The reference serves one engine per process behind an aiohttp app: an OpenAI-style speech endpoint that streams WAV
or raw PCM, a WebSocket that multiplexes several utterances ("contexts") on one connection, voice registration and a
health probe, with admission control (a bound on requests waiting for their first audio and a queue deadline) and a
cancel on every client disconnect.  This front keeps that wire protocol -- paths, JSON fields, the streaming WAV
header, the binary audio frame layout, error bodies and codes -- so a client of the reference talks to it unchanged,
and puts it in front of N replicas (one TickEngine per GPU), each driven by its own engine thread; a new request goes
to the least-loaded replica (router.Router) and stays there.

What a request carries differs in one place.  The layer under this front takes backbone token ids, so a request
either sends them (``"input_ids"``; on the WebSocket ``"text_ids"``) or sends text, which the server turns into ids
with the ``encode(text, lang, voice)`` callable it was built with (the reference's text normaliser, prompt builder and
tokenizer live there).  Voices are prefix token ids whose K/V each replica computes once (TickEngine.prepare_voice).
Audio is PCM s16le at 24 kHz mono; of the reference's encodings only the two that need no codec library (wav, pcm)
are produced, the others are refused with 400 naming the reason, as the reference refuses encoders it lacks.

Threads: the event loop never touches an engine.  It queues submissions, cancels and voice builds to a replica; the
replica's thread applies them between ticks, runs the tick (TickEngine.tick, or tick_pipelined for throughput) and
hands each tick's events to the loop with one call_soon_threadsafe per loop per tick.
"""
from __future__ import annotations

import asyncio
import base64
import collections
import concurrent.futures
import json
import math
import re
import struct
import threading
import time
import uuid

import numpy as np

from .config import FRAME, SAMPLE_RATE
from .router import Router

try:
    from aiohttp import WSMsgType, web
except ImportError:          # the engine layer does not need the front; the front raises when it is built
    web = None

SR = SAMPLE_RATE
MAX_FRAMES = 1500
SEED_MAX = 2 ** 63 - 1
LANGS = ("as", "bn", "en", "gu", "hi", "kn", "ml", "mr", "or", "pa", "ta", "te")
FORMATS = {"wav": "audio/wav", "pcm": "audio/pcm"}
REFUSED_FORMATS = {"mp3": "no MP3 encoder in this build", "opus": "no Opus encoder in this build",
                   "flac": "no FLAC encoder in this build", "aac": "no AAC encoder is bundled"}
OPENAI_VOICES = {"alloy", "ash", "ballad", "coral", "echo", "fable", "onyx", "nova", "sage", "shimmer", "verse",
                 "marin", "cedar"}
VOICE_ID_RE = re.compile(r"^[A-Za-z0-9][A-Za-z0-9_.\-]{0,63}$")
# Unicode blocks of the scripts the reference recognises, for requests that name no language
SCRIPT_BLOCKS = ((0x0900, 0x097F, "hi"), (0x0980, 0x09FF, "bn"), (0x0A00, 0x0A7F, "pa"), (0x0A80, 0x0AFF, "gu"),
                 (0x0B00, 0x0B7F, "or"), (0x0B80, 0x0BFF, "ta"), (0x0C00, 0x0C7F, "te"), (0x0C80, 0x0CFF, "kn"),
                 (0x0D00, 0x0D7F, "ml"))


# ------------------------------------------------------------------------------------------------ wire format
class ApiError(Exception):
    """A refused request: HTTP status, error code, message, offending field, Retry-After seconds."""

    def __init__(self, status, code, message, param=None, retry_after=None):
        super().__init__(message)
        self.status, self.code, self.message, self.param, self.retry_after = status, code, message, param, retry_after

    def body(self):
        kind = "invalid_request_error" if self.status < 500 else "server_error"
        return {"error": {"message": self.message, "type": kind, "code": self.code, "param": self.param}}

    def response(self):
        headers = {"Retry-After": str(self.retry_after)} if self.retry_after else None
        return web.json_response(self.body(), status=self.status, headers=headers)


def invalid(message, param=None):
    return ApiError(400, "invalid_request", message, param)


def wav_header(data_bytes=None, sr=SR):
    """RIFF/WAVE header of mono s16le PCM; without a length both sizes are 0xFFFFFFFF (a stream of unknown length)."""
    n = 0xFFFFFFFF if data_bytes is None else int(data_bytes)
    riff = 0xFFFFFFFF if data_bytes is None else 36 + n
    return (b"RIFF" + struct.pack("<I", riff) + b"WAVEfmt " +
            struct.pack("<IHHIIHH", 16, 1, 1, sr, sr * 2, 2, 16) + b"data" + struct.pack("<I", n))


def ws_audio_frame(context_id, pcm):
    """Binary WebSocket audio message: uint32-LE byte length of the context id, its UTF-8 bytes, then PCM s16le."""
    cid = context_id.encode()
    return struct.pack("<I", len(cid)) + cid + pcm


def guess_lang(text):
    """The language a request means when it names none: the most frequent script among its letters."""
    votes = collections.Counter()
    for ch in text:
        o = ord(ch)
        if o < 0x80:
            votes["en"] += ch.isalpha()
            continue
        for lo, hi, lang in SCRIPT_BLOCKS:
            if lo <= o <= hi:
                votes[lang] += 1
                break
    best = [lang for lang, n in votes.most_common() if n > 0]
    return best[0] if best else "en"


def _int(v):
    return isinstance(v, int) and not isinstance(v, bool)


def _num(v):
    return isinstance(v, (int, float)) and not isinstance(v, bool) and math.isfinite(v)


def parse_request(body, vocab, text_field, ids_field):
    """The fields one utterance request shares on HTTP and the WebSocket -> dict(text, ids, lang, voice, max_frames,
    sampling, normalize); ApiError(400) naming the field otherwise (the reference's ranges, maya3/server.py:190-261)."""
    out = {"text": None, "ids": None}
    ids = body.get(ids_field)
    text = body.get(text_field)
    if ids is not None:
        if (not isinstance(ids, list) or not ids or not all(_int(t) for t in ids)
                or not all(0 <= t < vocab for t in ids)):
            raise invalid(f"{ids_field} must be a non-empty list of token ids in [0, {vocab})", ids_field)
        out["ids"] = np.asarray(ids, np.int64)
    elif not isinstance(text, str) or not text.strip():
        raise invalid(f"{text_field} must be a non-empty string (or send {ids_field})", text_field)
    else:
        if len(text) > 4000:
            raise invalid(f"{text_field} is {len(text)} characters; the limit is 4000", text_field)
        out["text"] = text.strip()
    lang = body.get("language", body.get("lang"))
    if lang is None or lang == "auto":
        lang = guess_lang(out["text"] or "")
    elif not isinstance(lang, str) or lang.lower() not in LANGS:
        raise invalid(f"unsupported language {lang!r}; supported: {', '.join(LANGS)}", "language")
    out["lang"] = lang.lower()
    mf = body.get("max_frames")
    if mf is not None and (not _int(mf) or not 1 <= mf <= MAX_FRAMES):
        raise invalid(f"max_frames must be an integer in 1..{MAX_FRAMES} (80 ms frames)", "max_frames")
    out["max_frames"] = mf
    sp = {}
    checks = (("seed", lambda v: _int(v) and 0 <= v <= SEED_MAX, "an integer in 0..2^63-1"),
              ("temperature", lambda v: _num(v) and 0.1 <= v <= 1.5, "a number in 0.1..1.5"),
              ("top_k", lambda v: _int(v) and 1 <= v <= 2048, "an integer in 1..2048"),
              ("top_p", lambda v: _num(v) and 0 < v <= 1, "a number with 0 < top_p <= 1"),
              ("repetition_penalty", lambda v: _num(v) and 0 <= v <= 5, "a number in 0..5"))
    for key, ok, what in checks:
        v = body.get(key)
        if v is not None:
            if not ok(v):
                raise invalid(f"{key} must be {what}", key)
            sp[key] = v
    out["sampling"] = sp
    key = "normalize" if "normalize" in body else "normalise"
    norm = body.get(key, True)
    if norm is not None and not isinstance(norm, bool):
        raise invalid(f"{key} must be true or false", key)
    out["normalize"] = norm is not False
    voice = body.get("voice")
    if voice is not None and not isinstance(voice, str):
        raise invalid("voice must be a string (a registered voice id)", "voice")
    out["voice"] = voice or "plain"
    return out


# ------------------------------------------------------------------------------------------------ jobs
class Job:
    """One utterance as the event loop sees it: the engine's events (audio chunks, then one end or error) queued in
    order, the submit and first-audio times, and how much audio the client has not taken yet."""

    def __init__(self, loop, rid, max_lag_s=None, on_overflow=None):
        self.loop, self.rid = loop, rid
        self.items = collections.deque()
        self.ready = asyncio.Event()
        self.replica = None
        self.seat = None                   # the engine's Seat, set on the engine thread
        self.t_submit = time.perf_counter()
        self.t_first = None
        self.lag = 0                       # samples received and not yet taken
        self.max_lag = int(max_lag_s * SR) if max_lag_s else None
        self.on_overflow = on_overflow
        self.overflowed = False
        self.done = False                  # an end or error event arrived
        self.closed = False
        self.on_first = None               # called once, on the loop, when the first event arrives

    def put(self, kind, payload):          # event loop
        if self.closed:
            return
        if self.on_first is not None:
            cb, self.on_first = self.on_first, None
            cb(self)
        if kind == "audio":
            if self.t_first is None:
                self.t_first = time.perf_counter()
            self.lag += len(payload) // 2
            if self.max_lag is not None and self.lag > self.max_lag and not self.overflowed:
                self.overflowed = True
                self.cancel()
                if self.on_overflow is not None:
                    self.on_overflow()
        else:
            self.done = True
        self.items.append((kind, payload))
        self.ready.set()

    async def next(self, timeout=None):
        while not self.items:
            self.ready.clear()
            if timeout is None:
                await self.ready.wait()
            else:
                await asyncio.wait_for(self.ready.wait(), timeout)
        kind, payload = self.items.popleft()
        if kind == "audio":
            self.lag -= len(payload) // 2
        return kind, payload

    def take_audio(self, first, limit):
        """`first` joined with the audio already queued behind it (no waiting), up to `limit` samples."""
        parts, n = [first], len(first) // 2
        while n < limit and self.items and self.items[0][0] == "audio":
            _, p = self.items.popleft()
            self.lag -= len(p) // 2
            parts.append(p)
            n += len(p) // 2
        return b"".join(parts), n

    def interrupt(self):
        self.items.append(("interrupt", None))
        self.ready.set()

    def cancel(self):
        if not self.done and self.replica is not None:
            self.replica.cancel(self)

    def close(self):
        if not self.closed:
            self.cancel()
            self.closed = True


# ------------------------------------------------------------------------------------------------ replicas
class Replica:
    """One TickEngine driven by its own thread.  The event loop only queues work to it (submit, cancel, voices);
    the thread applies the queue between ticks, ticks while any request is active or waiting, and posts each tick's
    events to the jobs' loops in one batch per loop."""

    def __init__(self, engine, name="replica0", pipelined=False, idle_wait_s=0.02):
        self.engine, self.name, self.pipelined = engine, name, bool(pipelined)
        self.idle_wait_s = idle_wait_s
        self.voices = {}                   # voice id -> engine Voice (built on this replica's GPU)
        self.failed = None
        self._queue = collections.deque()
        self._wake = threading.Event()
        self._jobs = {}                    # id(seat) -> Job
        self._stopping = False
        self.queued = 0                    # submissions queued and not yet applied (load seen by the router)
        self.stats = collections.Counter()
        self._thread = threading.Thread(target=self._run, name=f"maya3-{name}", daemon=True)
        self._thread.start()

    # -- called from any thread
    def load(self):
        e = self.engine
        return len(e.active) + len(e.pending) + self.queued

    def submit(self, job, ids, max_frames, sampling, voice):
        job.replica = self
        self.queued += 1
        self._queue.append(("submit", job, (ids, max_frames, sampling, voice)))
        self._wake.set()

    def cancel(self, job):
        self._queue.append(("cancel", job, None))
        self._wake.set()

    def add_voice(self, vid, ids):
        """Build voice `vid` from prefix token ids on this replica (between ticks); a Future of its token count."""
        fut = concurrent.futures.Future()
        self._queue.append(("voice", fut, (vid, ids)))
        self._wake.set()
        return fut

    def drop_voice(self, vid):
        self._queue.append(("drop_voice", None, vid))
        self._wake.set()

    def health(self):
        e = self.engine
        return {"name": self.name, "device": str(getattr(e, "device", "")), "active": len(e.active),
                "pending": len(e.pending) + self.queued, "max_seats": e.cfg.max_seats, "ticks": e.stats["ticks"],
                "frames": e.stats["frames"], "pipelined": self.pipelined, "failed": self.failed,
                "voices": sorted(self.voices)}

    def close(self, timeout=10.0):
        self._stopping = True
        self._wake.set()
        self._thread.join(timeout)

    # -- engine thread
    def _run(self):
        import torch
        e = self.engine
        dev = getattr(e, "device", None)
        if dev is not None and getattr(dev, "type", None) == "cuda":
            torch.cuda.set_device(dev)
        try:
            with torch.inference_mode():
                while not self._stopping:
                    self._apply_queue()
                    if not (e.active or e.pending or getattr(e, "_inflight", None) is not None):
                        self._wake.wait(self.idle_wait_s)
                        self._wake.clear()
                        continue
                    out = e.tick_pipelined() if self.pipelined else e.tick()
                    self._post(out)
                if getattr(e, "_inflight", None) is not None:
                    self._post(e.flush())
        except Exception as exc:           # the engine is unusable: every open request ends with an error
            self.failed = f"{type(exc).__name__}: {exc}"
            self._fail_all("internal", f"engine failed: {self.failed}")

    def _apply_queue(self):
        e = self.engine
        while self._queue:
            op, obj, arg = self._queue.popleft()
            if op == "submit":
                self.queued -= 1
                ids, max_frames, sampling, voice = arg
                job = obj
                if job.closed:
                    continue
                try:
                    v = None
                    if voice not in (None, "plain"):
                        v = self.voices.get(voice)
                        if v is None:
                            raise ValueError(f"unknown voice {voice!r}")
                    seat = e.submit(ids, max_frames if max_frames is not None else MAX_FRAMES,
                                    rid=job.rid, sampling=sampling or None, voice=v)
                except ValueError as exc:
                    self._send({job.loop: [(job, "error", {"code": "invalid_request", "error": str(exc)})]})
                    continue
                job.seat = seat
                self._jobs[id(seat)] = job
                self.stats["submitted"] += 1
            elif op == "cancel":
                job = obj
                seat = job.seat
                if seat is not None and self._jobs.get(id(seat)) is job and e.cancel(seat):
                    del self._jobs[id(seat)]
                    self.stats["cancelled"] += 1
            elif op == "voice":
                vid, ids = arg
                try:
                    if getattr(e, "_inflight", None) is not None:
                        self._post(e.flush())      # the voice build runs eager steps in a free slot
                    self.voices[vid] = e.prepare_voice(ids)
                    obj.set_result(len(ids))
                except Exception as exc:
                    obj.set_exception(exc)
            elif op == "drop_voice":
                self.voices.pop(arg, None)

    def _post(self, out):
        """One tick's deliveries -> audio / end events, grouped by the jobs' event loops."""
        batches = collections.defaultdict(list)
        for s, code, cb0, pcm in out:
            job = self._jobs.get(id(s))
            if job is None:
                continue
            if pcm is not None:
                batches[job.loop].append((job, "audio", pcm.tobytes()))   # the view is reused two ticks later
            if s.stop is not None:
                info = {"reason": s.stop, "frames": s.frames, "audio_s": round(s.frames * FRAME / SR, 3)}
                batches[job.loop].append((job, "end", info))
                del self._jobs[id(s)]
                self.stats["completed"] += 1
        self._send(batches)

    def _fail_all(self, code, message):
        batches = collections.defaultdict(list)
        for job in self._jobs.values():
            batches[job.loop].append((job, "error", {"code": code, "error": message}))
        self._jobs.clear()
        while self._queue:
            op, obj, _ = self._queue.popleft()
            if op == "submit":
                batches[obj.loop].append((obj, "error", {"code": code, "error": message}))
            elif op == "voice":
                obj.set_exception(RuntimeError(message))
        self._send(batches)

    def _send(self, batches):
        for loop, items in batches.items():
            try:
                loop.call_soon_threadsafe(_put_batch, items)
            except RuntimeError:           # that loop is gone: its requests have no reader
                for job, _, _ in items:
                    if job.seat is not None and job.seat.stop is None:
                        self.cancel(job)


def _put_batch(items):
    for job, kind, payload in items:
        job.put(kind, payload)


# ------------------------------------------------------------------------------------------------ server
class Maya3Server:
    """The aiohttp front.  `replicas` are Replica objects (one per GPU); `encode(text, lang, voice)` turns a text
    request into backbone token ids (None: requests must send ids)."""

    def __init__(self, replicas, *, vocab, encode=None, max_pending=64, queue_deadline_ms=2000, ws_max_contexts=8,
                 ws_max_lag_s=20.0, http_max_lag_s=120.0, ws_send_queue=64, coalesce_ms=480, policy="least_loaded"):
        if web is None:
            raise RuntimeError("the HTTP / WebSocket front needs aiohttp")
        self.replicas = list(replicas)
        if not self.replicas:
            raise ValueError("at least one replica")
        self.vocab = int(vocab)
        self.encode = encode
        self.max_pending = int(max_pending)
        self.deadline = queue_deadline_ms / 1000.0
        self.ws_max_contexts = int(ws_max_contexts)
        self.ws_max_lag_s = ws_max_lag_s
        self.http_max_lag_s = http_max_lag_s
        self.ws_send_queue = int(ws_send_queue)
        self.coalesce = max(FRAME, int(coalesce_ms * SR / 1000))
        self.router = Router(len(self.replicas), policy)
        self.voices = {}                   # voice id -> {"id", "mode", "prefix_tokens"}
        self.waiting = set()               # jobs without their first event (admission control)
        self.sockets = 0
        self.stats = collections.Counter()

    # -- app
    def app(self):
        app = web.Application(client_max_size=8 * 1024 * 1024)
        app.on_cleanup.append(self._cleanup)
        r = app.router
        r.add_get("/health", self.health)
        r.add_get("/v1/models", self.models)
        r.add_post("/v1/audio/speech", self.speech)
        r.add_get("/v1/tts/stream", self.ws)
        r.add_get("/v1/voices", self.list_voices)
        r.add_post("/v1/voices", self.add_voice)
        r.add_delete("/v1/voices/{voice_id}", self.delete_voice)
        return app

    async def _cleanup(self, app):
        for job in list(self.waiting):
            job.close()

    def close(self):
        for r in self.replicas:
            r.close()

    # -- admission
    def _live(self):
        ok = [r for r in self.replicas if r.failed is None]
        if not ok:
            raise ApiError(503, "unavailable", "every engine replica has failed", retry_after=5)
        return ok

    def _resolve_voice(self, voice):
        if voice == "plain" or voice in self.voices:
            return voice
        low = voice.lower()
        for vid in self.voices:
            if vid.lower() == low:
                return vid
        if low in OPENAI_VOICES:
            return "plain"
        raise invalid(f"unknown voice {voice!r}; registered voices: {', '.join(['plain', *self.voices])}", "voice")

    def _ids(self, req):
        if req["ids"] is not None:
            return req["ids"]
        if self.encode is None:
            raise invalid("this server has no text front end: send backbone token ids", "input")
        try:
            ids = np.asarray(self.encode(req["text"], req["lang"], req["voice"]), np.int64)
        except ValueError as exc:
            raise invalid(str(exc), "input")
        if ids.ndim != 1 or len(ids) == 0:
            raise invalid("the text encodes to no tokens", "input")
        return ids

    def submit(self, req, rid, max_lag_s, on_overflow=None):
        """Admit one request and hand it to a replica: ApiError 503 when max_pending requests already wait for their
        first audio (maya3/server.py:516-535)."""
        live = self._live()
        if len(self.waiting) >= self.max_pending:
            self.stats["rejected_pending"] += 1
            raise ApiError(503, "overloaded", f"server overloaded: {len(self.waiting)} requests already waiting for "
                                              f"audio (max_pending={self.max_pending}); retry later", retry_after=1)
        voice = req["voice"] = self._resolve_voice(req["voice"])
        ids = self._ids(req)
        loads = [r.load() if r.failed is None else 1 << 30 for r in self.replicas]
        rep = self.replicas[self.router.route(loads)]
        if rep.failed is not None:         # round-robin landed on a failed replica: the least-loaded live one
            rep = min(live, key=lambda r: r.load())
        job = Job(asyncio.get_running_loop(), rid, max_lag_s, on_overflow)
        job.on_first = self.waiting.discard
        self.waiting.add(job)
        rep.submit(job, ids, req["max_frames"], req["sampling"], voice)
        self.stats["submitted"] += 1
        return job

    async def first_event(self, job, gone=None):
        """The job's first event within the queue deadline; past it the job is cancelled and ApiError 503 raised."""
        limit = job.t_submit + self.deadline
        while True:
            left = limit - time.perf_counter()
            if left <= 0:
                job.close()
                self.waiting.discard(job)
                self.stats["rejected_deadline"] += 1
                raise ApiError(503, "overloaded", f"no audio within the queue deadline of {self.deadline * 1e3:.0f} "
                                                  "ms; retry later", retry_after=1)
            try:
                return await job.next(timeout=min(left, 0.2))
            except asyncio.TimeoutError:
                if gone is not None and gone():
                    job.close()
                    self.waiting.discard(job)
                    raise ConnectionResetError("client went away")

    # -- HTTP
    async def health(self, request):
        reps = [r.health() for r in self.replicas]
        ready = any(r["failed"] is None for r in reps)
        body = {"ready": ready, "replicas": reps,
                "server": {"waiting": len(self.waiting), "ws_sockets": self.sockets, "max_pending": self.max_pending,
                           "queue_deadline_ms": self.deadline * 1e3, "formats": list(FORMATS),
                           "text_front_end": self.encode is not None, **self.stats}}
        return web.json_response(body, status=200 if ready else 503)

    async def models(self, request):
        return web.json_response({"object": "list", "data": [{"id": "maya3", "object": "model", "owned_by": "maya"}]})

    async def _body(self, request):
        try:
            body = await request.json()
        except Exception:
            raise invalid("request body must be a JSON object")
        if not isinstance(body, dict):
            raise invalid("request body must be a JSON object")
        return body

    async def speech(self, request):
        try:
            return await self._speech(request)
        except ApiError as exc:
            return exc.response()

    async def _speech(self, request):
        self._live()
        body = await self._body(request)
        req = parse_request(body, self.vocab, "input", "input_ids")
        fmt = body.get("response_format", "wav") or "wav"
        if not isinstance(fmt, str) or fmt.lower() not in FORMATS:
            why = REFUSED_FORMATS.get(fmt.lower()) if isinstance(fmt, str) else None
            raise invalid(f"response_format {fmt!r}" + (f" is not supported ({why})" if why else "") +
                          f"; use one of: {', '.join(FORMATS)}", "response_format")
        fmt = fmt.lower()
        speed = body.get("speed", 1.0)
        if not _num(speed) or float(speed) != 1.0:
            raise invalid("speed must be 1.0 (speed control is not supported)", "speed")
        sfmt = body.get("stream_format", "audio") or "audio"
        if sfmt not in ("audio", "sse"):
            raise invalid("stream_format must be 'audio' or 'sse'", "stream_format")
        rid = f"h-{uuid.uuid4().hex[:16]}"
        resp = None

        def abort():
            if request.transport is not None:
                request.transport.abort()
        job = self.submit(req, rid, self.http_max_lag_s, on_overflow=abort)
        gone = lambda: request.transport is None or request.transport.is_closing()
        try:
            kind, payload = await self.first_event(job, gone)
            if kind == "error":
                code = payload.get("code") or "unavailable"
                raise ApiError(400 if code == "invalid_request" else 503, code, payload.get("error") or code)
            headers = {"Content-Type": "text/event-stream" if sfmt == "sse" else FORMATS[fmt],
                       "X-Sample-Rate": str(SR), "X-Channels": "1", "X-Encoding": "pcm_s16le",
                       "X-Maya3-Language": req["lang"], "X-Maya3-Voice": self._resolve_voice(req["voice"]),
                       "X-Maya3-Normalized": "1" if (req["normalize"] and req["ids"] is None and self.encode) else "0",
                       "X-Request-Id": rid, "Cache-Control": "no-store"}
            resp = web.StreamResponse(headers=headers)
            resp.enable_chunked_encoding()
            await resp.prepare(request)

            async def send(data):
                if sfmt == "sse":
                    data = b"data: " + json.dumps({"type": "speech.audio.delta",
                                                   "audio": base64.b64encode(data).decode()}).encode() + b"\n\n"
                await resp.write(data)
            if fmt == "wav":
                await send(wav_header())
            while True:
                if kind == "audio":
                    data, _ = job.take_audio(payload, self.coalesce)
                    await send(data)
                elif kind == "end":
                    if sfmt == "sse":
                        usage = {k: payload.get(k) for k in ("audio_s", "frames", "reason")}
                        await resp.write(b"data: " + json.dumps({"type": "speech.audio.done",
                                                                 "usage": usage}).encode() + b"\n\n")
                    await resp.write_eof()
                    self.stats["completed"] += 1
                    return resp
                elif kind == "error":      # never close a failed utterance as if it had ended
                    self.stats["aborted_midstream"] += 1
                    abort()
                    return resp
                else:
                    abort()
                    return resp
                kind, payload = await job.next()
        except ConnectionResetError:
            self.stats["client_gone"] += 1
            return resp if resp is not None else web.Response(status=499)
        except ApiError:
            if resp is not None:
                abort()
                return resp
            raise
        finally:
            if job.overflowed:
                self.stats["slow_consumer"] += 1
            job.close()

    # -- voices
    async def list_voices(self, request):
        return web.json_response({"voices": [{"id": "plain", "mode": "plain"}, *self.voices.values()]})

    async def add_voice(self, request):
        try:
            self._live()
            body = await self._body(request)
            vid = body.get("voice_id")
            if not isinstance(vid, str) or not VOICE_ID_RE.match(vid) or vid == "plain":
                raise invalid("voice_id must match [A-Za-z0-9][A-Za-z0-9_.-]{0,63} and not be 'plain'", "voice_id")
            if vid in self.voices and not body.get("replace", False):
                raise ApiError(409, "voice_exists", f"voice {vid!r} exists; send replace: true to overwrite",
                               "voice_id")
            ids = body.get("prefix_ids")
            if ids is None and isinstance(body.get("ref_text"), str) and self.encode is not None:
                ids = [int(t) for t in self.encode(body["ref_text"], body.get("lang") or "en", "plain")]
            if (not isinstance(ids, list) or not ids or not all(_int(t) and 0 <= t < self.vocab for t in ids)):
                raise invalid("prefix_ids must be a non-empty list of backbone token ids", "prefix_ids")
            t0 = time.perf_counter()
            futs = [asyncio.wrap_future(r.add_voice(vid, np.asarray(ids, np.int64))) for r in self._live()]
            try:
                await asyncio.gather(*futs)
            except (ValueError, RuntimeError) as exc:
                raise invalid(str(exc), "prefix_ids")
            self.voices[vid] = {"id": vid, "mode": "prefix", "prefix_tokens": len(ids)}
            return web.json_response({**self.voices[vid], "register_s": round(time.perf_counter() - t0, 3)},
                                     status=201)
        except ApiError as exc:
            return exc.response()

    async def delete_voice(self, request):
        vid = request.match_info["voice_id"]
        if vid not in self.voices:
            return ApiError(404, "voice_not_found", f"no voice {vid!r}", "voice_id").response()
        del self.voices[vid]
        for r in self.replicas:
            r.drop_voice(vid)
        return web.json_response({"id": vid, "deleted": True})

    # -- WebSocket
    async def ws(self, request):
        ws = web.WebSocketResponse(heartbeat=30, max_msg_size=64 * 1024)
        await ws.prepare(request)
        sock = _Socket(self, ws, request)
        self.sockets += 1
        sock.start()
        sock.put({"type": "metadata", "sample_rate": SR, "encoding": "pcm_s16le", "channels": 1,
                  "max_contexts": self.ws_max_contexts, "languages": list(LANGS)})
        try:
            async for msg in ws:
                if msg.type == WSMsgType.TEXT:
                    sock.on_text(msg.data)
                elif msg.type == WSMsgType.BINARY:
                    sock.error(None, "invalid_request", "send JSON text messages (speak / cancel / ping)")
                elif msg.type == WSMsgType.ERROR:
                    break
        finally:
            self.sockets -= 1
            await sock.close()
        return ws


class _Context:
    """One utterance on a socket."""
    __slots__ = ("cid", "job", "task", "binary", "stop", "samples")

    def __init__(self, cid, binary):
        self.cid, self.binary = cid, binary
        self.job = self.task = self.stop = None
        self.samples = 0


class _Socket:
    """One WebSocket: the reader (the handler's loop), one pump task per context, and one writer draining a bounded
    outgoing queue (audio waits for room; control messages never do)."""

    def __init__(self, srv, ws, request):
        self.srv, self.ws, self.request = srv, ws, request
        self.contexts = {}
        self.out = collections.deque()     # (context id or None, is audio, message)
        self.wake = asyncio.Event()
        self.room = asyncio.Event()
        self.room.set()
        self.closed = False
        self.writer = None

    def start(self):
        self.writer = asyncio.create_task(self._write())

    def put(self, msg, cid=None, audio=False):
        self.out.append((cid, audio, msg))
        self.wake.set()

    def error(self, cid, code, message):
        self.put({"type": "error", "context_id": cid, "code": code, "error": message})

    async def _write(self):
        try:
            while True:
                while not self.out:
                    self.wake.clear()
                    await self.wake.wait()
                _, _, msg = self.out.popleft()
                if len(self.out) < self.srv.ws_send_queue:
                    self.room.set()
                if self.ws.closed:
                    continue
                try:
                    if isinstance(msg, bytes):
                        await asyncio.wait_for(self.ws.send_bytes(msg), 15.0)
                    else:
                        await asyncio.wait_for(self.ws.send_str(json.dumps(msg)), 15.0)
                except (asyncio.TimeoutError, ConnectionResetError, RuntimeError):
                    self._drop()
                    return
        except asyncio.CancelledError:
            pass

    def _drop(self):
        self.closed = True
        self.room.set()
        for ctx in list(self.contexts.values()):
            self._stop(ctx, "disconnected")
        if self.request.transport is not None:
            self.request.transport.abort()

    def on_text(self, data):
        cid = None
        try:
            try:
                msg = json.loads(data)
            except ValueError:
                raise invalid("message is not valid JSON")
            if not isinstance(msg, dict):
                raise invalid("message must be a JSON object")
            cid = msg.get("context_id")
            if cid is not None and (not isinstance(cid, str) or not 1 <= len(cid) <= 128):
                cid = None
                raise invalid("context_id must be a string of 1-128 characters", "context_id")
            kind = msg.get("type")
            if kind == "ping":
                self.put({"type": "pong", **({"context_id": cid} if cid else {})})
            elif kind == "cancel":
                ctx = self.contexts.get(cid)
                if ctx is not None:
                    self._stop(ctx, "cancelled")
            elif kind == "speak":
                self._speak(cid, msg)
            else:
                raise invalid("unknown message type; use speak, cancel or ping", "type")
        except ApiError as exc:
            self.error(cid, exc.code, exc.message)

    def _speak(self, cid, msg):
        srv = self.srv
        if cid is None:
            raise invalid("speak needs a context_id", "context_id")
        if cid in self.contexts:
            raise invalid(f"context {cid!r} is still active; use a new context_id", "context_id")
        if len(self.contexts) >= srv.ws_max_contexts:
            raise ApiError(429, "too_many_contexts", f"at most {srv.ws_max_contexts} concurrent contexts per "
                                                     "connection")
        srv._live()
        req = parse_request(msg, srv.vocab, "text", "text_ids")
        binary = msg.get("binary", False)
        if not isinstance(binary, bool):
            raise invalid("binary must be true or false", "binary")
        ctx = _Context(cid, binary)
        ctx.job = srv.submit(req, f"w-{uuid.uuid4().hex[:12]}", srv.ws_max_lag_s,
                             on_overflow=lambda: self._stop(ctx, "slow_consumer"))
        self.contexts[cid] = ctx
        ctx.task = asyncio.create_task(self._pump(ctx))

    def _stop(self, ctx, reason):
        if ctx.stop is None:
            ctx.stop = reason
            ctx.job.close()
            ctx.job.interrupt()
            if any(c == ctx.cid and a for c, a, _ in self.out):     # its audio not yet sent is dropped
                self.out = collections.deque(x for x in self.out if not (x[0] == ctx.cid and x[1]))
            self.room.set()

    async def _send_audio(self, ctx, msg):
        while len(self.out) >= self.srv.ws_send_queue and not self.closed and ctx.stop is None:
            self.room.clear()
            await self.room.wait()
        if self.closed or ctx.stop is not None:
            return False
        self.put(msg, ctx.cid, True)
        return True

    def _ttfa(self, job):
        return round((job.t_first - job.t_submit) * 1e3, 1) if job.t_first else None

    async def _pump(self, ctx):
        srv, cid, job = self.srv, ctx.cid, ctx.job
        try:
            try:
                kind, payload = await srv.first_event(job)
            except ApiError as exc:
                self.error(cid, exc.code, exc.message)
                return
            while ctx.stop is None:
                if kind == "audio":
                    pcm, n = job.take_audio(payload, srv.coalesce)
                    msg = (ws_audio_frame(cid, pcm) if ctx.binary else
                           {"type": "audio", "context_id": cid, "audio": base64.b64encode(pcm).decode()})
                    if await self._send_audio(ctx, msg):
                        ctx.samples += n
                elif kind == "end":
                    self.put({"type": "end", "context_id": cid, "reason": payload.get("reason"),
                              "frames": payload.get("frames"), "audio_s": payload.get("audio_s"),
                              "ttfa_ms": self._ttfa(job)})
                    srv.stats["completed"] += 1
                    return
                elif kind == "error":
                    self.error(cid, payload.get("code") or "internal", payload.get("error") or "internal")
                    return
                kind, payload = await job.next()
            if ctx.stop == "cancelled":
                self.put({"type": "end", "context_id": cid, "reason": "cancelled", "frames": ctx.samples // FRAME,
                          "audio_s": round(ctx.samples / SR, 3), "ttfa_ms": self._ttfa(job)})
                srv.stats["cancelled"] += 1
            elif ctx.stop == "slow_consumer":
                srv.stats["slow_consumer"] += 1
                self.error(cid, "slow_consumer", f"client fell more than {srv.ws_max_lag_s:.0f} s of audio behind; "
                                                 "request cancelled")
        except asyncio.CancelledError:
            pass
        finally:
            job.close()
            srv.waiting.discard(job)
            if self.contexts.get(cid) is ctx:
                del self.contexts[cid]

    async def close(self):
        self.closed = True
        self.room.set()
        ctxs = list(self.contexts.values())
        for ctx in ctxs:
            self._stop(ctx, "disconnected")
            ctx.task.cancel()
        await asyncio.gather(*(c.task for c in ctxs), return_exceptions=True)
        if self.writer is not None:
            self.writer.cancel()
            await asyncio.gather(self.writer, return_exceptions=True)


def serve(server, host="127.0.0.1", port=8080):
    """Run the front until interrupted (aiohttp's runner); the replicas' threads stop with it."""
    try:
        web.run_app(server.app(), host=host, port=port, access_log=None, handler_cancellation=True)
    finally:
        server.close()


__all__ = ["ApiError", "Job", "Maya3Server", "Replica", "serve", "wav_header", "ws_audio_frame", "parse_request",
           "guess_lang"]
