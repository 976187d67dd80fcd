"""TickEngine: the per-tick seat loop of maya3/engine.py (Engine._admit/_bind/_tick/_release) on the native tick.

What the reference's engine thread does per 80 ms frame for all seats -- admit new requests into free slots with an
inline prefill of their prompt, one backbone step over decode + prefill rows, the cb0 sampler, the depth loop, the
Mimi frame, one device->host readout and one sync (maya3/engine.py:514-630) -- is here one ``m3_tick_run`` call
replayed from a CUDA graph per (row bucket, seat bucket, context bucket), plus the host bookkeeping around it.  With
``TickConfig.guards`` set, the loop guard and frame cap (maya3/engine.py:571-617) run inside the tick on the device
(guards.py); their text-derived inputs (a piece's cap from the duration prior, its suspend windows) come with the
request.  Text normalisation, prompt building and voices stay above this layer; a request here is a prompt of
backbone token ids and a frame budget.
"""
from __future__ import annotations

import dataclasses
import itertools
from typing import Optional

import numpy as np
import torch

from . import _lib as L
from .backbone import StaticBackbone
from .codec import StaticMimi
from .config import FRAME, Maya3Geom
from .depth import FastDepth
from .guards import VERDICTS, DeviceGuards, GuardConfig, merge_windows, split_code
from .sampler import Cb0Sampler

BUCKETS = (1, 2, 4, 8, 16, 24, 32, 48, 64, 80, 96, 112, 128, 160, 192, 224, 256)        # maya3/engine.py:44
ROW_BUCKETS = (1, 2, 4, 8, 16, 24, 32, 48, 64, 80, 96, 112, 128, 160, 192, 224, 256, 320, 384, 448, 512, 640,
               768, 1024)
CTX = (256, 512, 768, 1024, 1536, 2048, 3072)                                               # maya3/engine.py:191
REASONS = {1: "aeos", 2: "aeos_argmax", 3: "aeos_tau", 4: "aeos_hazard"}                    # maya3/engine.py:46
FROM_FEEDBACK = -2   # plan source of a decode row: its seat's feedback vector


@dataclasses.dataclass
class TickConfig:
    """The EngineConfig fields this layer uses (maya3/engine.py:49-79)."""
    max_seats: int = 16
    capacity: int = 2048
    temp: float = 0.7                 # depth sampler
    top_k: int = 64
    cb0_temp: float = 0.9
    cb0_top_k: int = 64
    cb0_top_p: float = 1.0
    cb0_rep: float = 0.8
    cb0_rep_win: int = 12
    max_inline_rows: int = 512        # prefill rows folded into one tick
    max_admit_per_tick: int = 8
    busy_frac: float = 0.75
    busy_admit: int = 4
    seed: int = 20261024
    stops: bool = True                # False: forced lengths, stop codes are ignored
    min_frames: int = 4
    greedy: bool = False              # depth levels by argmax (FastDepth greedy); cb0 greedy is cb0_top_k = 1
    use_graphs: bool = True
    # SMs the codec part's persistent SEANet kernels spread over when it runs beside the next tick's main part
    # (tick_pipelined; None: a quarter of the device's, 0: all).  Measured on one box: decode ticks 6.82 ms with all
    # SMs, 6.74 ms with a quarter.  A synchronous tick runs its codec part alone, on every SM.
    codec_sms: Optional[int] = None
    guards: Optional[GuardConfig] = None   # loop guard + frame cap on the device (maya3/engine.py:69); None = off


@dataclasses.dataclass
class Voice:
    """A voice's backbone prefix (maya3/engine.py:259-283 prepare_voice): its token ids and the packed K/V store of
    those positions, computed once and installed into each of its requests' slots with one launch."""
    ids: np.ndarray
    store: torch.Tensor
    length: int


@dataclasses.dataclass
class Seat:
    rid: object
    prompt: np.ndarray
    max_frames: int
    seed: int
    slot: int = -1
    frames: int = 0
    new: bool = True
    stop: Optional[str] = None
    inline: Optional[np.ndarray] = None   # the part of the prompt prefilled inline in the admission tick
    cap: int = 0                          # frame cap of the piece (_Seat.cap; the frame budget unless the caller's
    loose_cap: int = 0                    # duration prior lowers it) and the prior-free cap (_Seat.loose_cap)
    suspend: tuple = ()                   # inclusive frame windows with no loop action (_Seat.suspend)
    n_boost: int = 0                      # EOS boosts the loop guard applied (_Seat.n_boost)
    voice: Optional[Voice] = None         # prefix KV installed at bind; the prompt follows it
    sampling: dict = dataclasses.field(default_factory=dict)   # per-request cb0 sampling (check_sampling)


@dataclasses.dataclass
class TickPlan:
    plan: np.ndarray
    rows: int
    seats: int
    ctx: int
    dec: list
    new: list
    keys: int = 0


def _bucket(values, need, what):
    for b in values:
        if b >= need:
            return b
    raise ValueError(f"{what} {need} exceeds largest bucket {values[-1]}")


def admission_cap(n_active: int, cfg: "TickConfig") -> int:
    """How many pending requests one tick may admit (maya3/engine.py:451-454): max_admit_per_tick, or busy_admit once
    more than busy_frac of the seats are taken."""
    cap = cfg.max_admit_per_tick
    if n_active > cfg.busy_frac * cfg.max_seats:
        cap = min(cap, cfg.busy_admit)
    return cap


def frame_budget(prompt_len: int, max_frames: int, capacity: int) -> int:
    """A request's frame budget inside the KV capacity (maya3/engine.py:465-472): prompt + frames + 2 must fit; a
    budget clipped below 8 frames rejects the request."""
    if prompt_len + max_frames + 2 > capacity:
        max_frames = capacity - prompt_len - 2
        if max_frames < 8:
            raise ValueError(f"prompt of {prompt_len} tokens leaves no room in KV capacity {capacity}")
    return max_frames


SAMPLING_KEYS = ("seed", "temperature", "top_k", "top_p", "repetition_penalty")


def check_sampling(sp) -> dict:
    """A request's cb0 sampling overrides (maya3/engine.py:110-125): only the keys of SAMPLING_KEYS, None values
    dropped, each inside the reference's range; ValueError otherwise."""
    if not sp:
        return {}
    unknown = set(sp) - set(SAMPLING_KEYS)
    if unknown:
        raise ValueError(f"unknown sampling keys {sorted(unknown)}; allowed {sorted(SAMPLING_KEYS)}")
    out = {k: v for k, v in sp.items() if v is not None}
    limits = {"temperature": (0.05, 2.0), "top_k": (1, 2049), "repetition_penalty": (0.0, 5.0)}
    for k, (lo, hi) in limits.items():
        if k in out and not lo <= float(out[k]) <= hi:
            raise ValueError(f"{k} must be in [{lo}, {hi}]")
    if "top_p" in out and not 0.0 < float(out["top_p"]) <= 1.0:
        raise ValueError("top_p must be in (0, 1]")
    if "seed" in out and (isinstance(out["seed"], bool) or int(out["seed"]) < 0):
        raise ValueError("seed must be a non-negative integer")
    return out


def plan_layout(dec, new, lengths, row_buckets, seat_buckets, ctx_buckets, dummy):
    """The m3_tick_run plan of one tick: rows = one decode row per `dec` slot, then each admitted seat's inline prompt
    rows at consecutive offsets; then per seat (decode seats first) its slot and the row holding its last position.

    dec: decode slots; new: [(slot, inline token ids)]; lengths: the slots' current KV lengths (host mirror).
    Returns (plan int64 [4 * rb + 2 * sb], rb, sb, cb, keys): the row / seat / context buckets and the number of keys
    one attention launch reads (decode rows: length + 1; prefill row at offset o: o + 1; padding rows: 1)."""
    nd = len(dec)
    n_rows = nd + sum(len(t) for _, t in new)
    rb = _bucket(row_buckets, max(n_rows, 1), "rows")
    sb = _bucket(seat_buckets, max(nd + len(new), 1), "seats")
    dl = [lengths[s] for s in dec]
    need = max(max(dl, default=0) + 1, max((lengths[s] + len(t) for s, t in new), default=1))
    cb = _bucket(ctx_buckets, need, "context")
    keys = (sum(dl) + nd + sum(lengths[s] * len(t) + len(t) * (len(t) + 1) // 2 for s, t in new)
            + (rb - n_rows))
    p = np.zeros(4 * rb + 2 * sb, np.int64)
    r_slot, r_off, r_real, r_src = p[:rb], p[rb:2 * rb], p[2 * rb:3 * rb], p[3 * rb:4 * rb]
    s_slot, s_row = p[4 * rb:4 * rb + sb], p[4 * rb + sb:]
    r_slot[:] = dummy
    r_src[:] = -1
    s_slot[:] = dummy
    if nd:
        r_slot[:nd] = dec
        r_real[:nd] = 1
        r_src[:nd] = FROM_FEEDBACK
        s_slot[:nd] = dec
        s_row[:nd] = np.arange(nd)
    at = nd
    for j, (slot, toks) in enumerate(new):
        P = len(toks)
        r_slot[at:at + P] = slot
        r_off[at:at + P] = np.arange(P)
        r_real[at:at + P] = 1
        r_src[at:at + P] = toks
        at += P
        s_slot[nd + j] = slot
        s_row[nd + j] = at - 1
    return p, rb, sb, cb, keys


class _Graph:
    """The main part of a tick (backbone through the feedback write-back) for one bucket."""
    __slots__ = ("graph", "plan", "staging", "evt", "launches")


class _Codec:
    """The codec part of a tick (Mimi frame + packed readout) for one seat bucket and codec input set."""
    __slots__ = ("graph", "packed", "launches", "beside")


class TickEngine:
    def __init__(self, geom: Maya3Geom, weights: dict, config: TickConfig = None, device=None):
        self.cfg = cfg = config or TickConfig()
        self.geom = g = geom
        self.device = dev = (torch.device(device) if device is not None
                             else torch.device("cuda", torch.cuda.current_device()))
        n = cfg.max_seats
        self.buckets = tuple(b for b in BUCKETS if b < n) + (next((b for b in BUCKETS if b >= n), n),)
        rows = tuple(b for b in ROW_BUCKETS if b <= self.buckets[-1] + cfg.max_inline_rows)
        self.row_buckets = rows + tuple(b for b in ROW_BUCKETS if b > rows[-1])[:1]
        self.max_rows = self.row_buckets[-1]
        self.ctx_buckets = tuple(c for c in CTX if c < cfg.capacity) + (cfg.capacity,)
        self.backbone = StaticBackbone(weights, n, capacity=cfg.capacity, batch_buckets=self.row_buckets,
                                       ctx_buckets=self.ctx_buckets, use_graphs=False, geom=g.backbone, device=dev)
        self.cb0 = Cb0Sampler(weights["cb0_head.weight"], n, max_rows=self.buckets[-1], temp=cfg.cb0_temp,
                              top_k=cfg.cb0_top_k, top_p=cfg.cb0_top_p, rep=cfg.cb0_rep, rep_win=cfg.cb0_rep_win,
                              device=dev)
        self.depth = FastDepth(weights, n, temp=cfg.temp, top_k=cfg.top_k, batch_buckets=self.buckets,
                               seed=cfg.seed + 1, greedy=cfg.greedy, geom=g.depth, device=dev)
        self.codec = StaticMimi(weights, n, batch_buckets=self.buckets, geom=g.mimi, device=dev)
        # the codec's SM budget when its part runs beside the next tick's main part (pipelined ticks); a synchronous
        # tick runs it alone, on every SM
        self._codec_sms = cfg.codec_sms if cfg.codec_sms is not None else \
            torch.cuda.get_device_properties(dev).multi_processor_count // 4
        D = g.backbone.hidden
        with torch.inference_mode():
            self.embed = weights["model.embed_tokens.weight"].detach().to(dev, torch.bfloat16).contiguous()
            self.feedback = torch.zeros(n + 1, D, device=dev, dtype=torch.bfloat16)
            # one voice: every seat's speaker constant is FastDepth.set_speaker of the learned null memory
            self.depth.set_speaker(0, weights["depth.null_mem"].reshape(1, 1, -1), torch.ones(1, 1, dtype=torch.bool))
            self.voice_const = self.depth.cross_const[0].clone()
        self.spf = g.mimi.samples_per_frame
        tc = L.TickConfig(self.backbone._handle, self.cb0._handle, self.depth._handle, self.codec._handle,
                          self.embed.data_ptr(), self.embed.shape[0], self.feedback.data_ptr(), D, self.max_rows,
                          self.buckets[-1], g.depth.n_q, self.spf, n)
        h = L.vp()
        L.check(L.load().m3_tick_create(tc, h), "m3_tick_create")
        self._handle = h
        self.guards = None
        if cfg.guards is not None:
            self.guards = DeviceGuards(cfg.guards, n, self.cb0.aeos_bias)
            L.check(L.load().m3_tick_set_guard(h, self.guards.c_cfg, self.guards.c_state), "m3_tick_set_guard")
        self.free = list(range(n))[::-1]
        self.active: list[Seat] = []
        self.pending: list[Seat] = []
        self._rng = np.random.default_rng(cfg.seed)
        self._ids = itertools.count()
        self.graphs = {}
        self.codec_graphs = {}
        self.pool = None
        # the codec part of tick t runs on its own stream beside the main part of tick t + 1; its inputs alternate
        # between two sets, and a set is restaged only after the codec part that last read it has finished
        self.codec_stream = torch.cuda.Stream(device=dev)
        self._set = 0
        self._set_free = [None, None]
        # two pinned readout buffers, used in turn: a tick's PCM views stay valid while the next tick is in flight
        self._hosts = [torch.empty(self.buckets[-1], 2 + self.spf // 4, dtype=torch.int64).pin_memory()
                       for _ in range(2)]
        self._flip = 0
        self._inflight = None       # (plan, host rows, event) of the pipelined tick not yet delivered
        self._early = set()         # ids of seats whose slots were released before their last tick was read
        self._readout = None
        c, d = self.cb0, self.depth
        self._slot_state = L.SlotState(
            c.frames_t.data_ptr(), c.min_t.data_ptr(), c.hazard_t.data_ptr(), c.aeos_bias.data_ptr(),
            c.seed_t.data_ptr(), c.ctr_t.data_ptr(), c.hist_t.data_ptr(), c.hist_t.shape[1], c.temp_t.data_ptr(),
            c.topk_t.data_ptr(), c.topp_t.data_ptr(), c.rep_t.data_ptr(), d.row_seed.data_ptr(), d.row_ctr.data_ptr(),
            d.cross_const.data_ptr(), d.cross_const[0].numel(), self.backbone.lengths.data_ptr(), n)
        self.stats = {"ticks": 0, "admitted": 0, "completed": 0, "frames": 0, "prefill_rows": 0,
                      "eager_prefill_rows": 0}

    def close(self):
        if getattr(self, "_handle", None):
            torch.cuda.synchronize(self.device)     # the codec stream may still run the last tick's codec part
            self.graphs.clear()
            self.codec_graphs.clear()
            L.load().m3_tick_destroy(self._handle)
            self._handle = None
            for c in (self.backbone, self.cb0, self.depth, self.codec):
                c.close()

    def device_status(self, clear=True) -> int:
        torch.cuda.synchronize(self.device)     # the codec stream's last tick included
        s = L.i32(0)
        L.check(L.load().m3_tick_status(self._handle, s, int(clear)), "m3_tick_status")
        return int(s.value)

    # ---------------------------------------------------------------- requests
    @torch.inference_mode()
    def prepare_voice(self, prefix_ids) -> Voice:
        """maya3/engine.py:259-283: compute a voice prefix's backbone K/V once (here with this engine's own prefill,
        in a free slot, between ticks) for requests that then skip those positions (maya3/engine.py:488-491)."""
        ids = np.asarray(prefix_ids, np.int64)
        if ids.ndim != 1 or len(ids) == 0 or len(ids) >= self.cfg.capacity:
            raise ValueError("a voice prefix is a non-empty 1-D array of token ids shorter than the KV capacity")
        if not self.free:
            raise RuntimeError("prepare_voice needs a free slot")
        slot = self.free[-1]
        x = self.embed[torch.from_numpy(ids).to(self.device)]
        store = self.backbone.build_prefix(slot, x, chunk=self.cfg.max_inline_rows)
        return Voice(ids, store, len(ids))

    def submit(self, prompt_ids, max_frames, rid=None, seed=None, cap=None, loose_cap=None, suspend=(),
               voice: Optional[Voice] = None, sampling=None) -> Seat:
        """Queue a request: backbone token ids of its prompt and a frame budget (its length when stops=False), clipped
        to the KV capacity as the reference does (a budget below 8 frames rejects the request).  With guards on,
        `cap` is the piece's frame cap from the caller's duration prior and `loose_cap` its prior-free cap
        (maya3/engine.py:405-411, Engine._plan; both default to the budget), `suspend` its loop-guard suspend windows.
        With a `voice` (prepare_voice), the prompt is what follows the voice prefix.  `sampling` holds the request's
        cb0 overrides (check_sampling; the depth levels keep the engine's temperature and top-k); its "seed" derives
        the request's sampler streams as the reference's bind does for a one-piece request (maya3/engine.py:430-433),
        where `seed` is the stream seed itself."""
        prompt = np.asarray(prompt_ids, np.int64)
        if prompt.ndim != 1 or len(prompt) == 0:
            raise ValueError("prompt must be a non-empty 1-D array of token ids")
        sp = check_sampling(sampling)
        pre = voice.length if voice is not None else 0
        frames = frame_budget(pre + len(prompt), int(max_frames), self.cfg.capacity)
        if "seed" in sp:
            seed = (int(sp.pop("seed")) * 1000003) % (2 ** 31 - 1)
        else:
            seed = int(seed) if seed is not None else int(self._rng.integers(1, 2 ** 31 - 1))
        s = Seat(rid if rid is not None else next(self._ids), prompt, frames, seed)
        s.sampling = sp
        s.loose_cap = frames if loose_cap is None else min(int(loose_cap), frames)
        s.cap = min(s.loose_cap if cap is None else int(cap), frames)
        s.suspend = tuple(suspend)
        s.voice = voice
        if self.guards is not None and len(merge_windows(s.suspend)) > self.guards.cfg.max_windows:
            raise ValueError(f"more than {self.guards.cfg.max_windows} disjoint suspend windows")
        self.pending.append(s)
        return s

    def _bind(self, s: Seat):
        """maya3/engine.py:420-447: claim a slot and reset its per-slot state on the device."""
        self._claim(s)
        self.reset_slot(s)

    def _claim(self, s: Seat):
        s.slot = self.free.pop()
        self.backbone.lengths_cpu[s.slot] = s.voice.length if s.voice is not None else 0

    @torch.inference_mode()
    def reset_slot(self, s: Seat):
        """The device half of binding a seat: sampler, depth, codec and backbone state of its slot (stream-ordered,
        no host sync)."""
        slot = s.slot
        c, sp, cfg = self.cb0, s.sampling, self.cfg
        # maya3/engine.py:427-446: sampler, depth stream and backbone state of the slot in one launch; the request's
        # cb0 sampling overrides (or the engine's values) and the depth stream seed derived from its seed
        rep = float(sp["repetition_penalty"] if sp.get("repetition_penalty") is not None else cfg.cb0_rep)
        init = L.SlotInit(slot, s.seed, (s.seed * 69069 + 1) % (2 ** 31 - 1), cfg.min_frames,
                          int(sp.get("top_k") or cfg.cb0_top_k), 0, float(sp.get("temperature") or cfg.cb0_temp),
                          float(sp.get("top_p") or cfg.cb0_top_p), rep, self.voice_const.data_ptr())
        L.check(L.load().m3_slot_reset(self._slot_state, init, L.stream_ptr()), "m3_slot_reset")
        if float(sp.get("top_p") or 1.0) < 1.0:
            c.any_top_p = True
        if sp.get("repetition_penalty"):
            c.any_rep = True
        with torch.cuda.stream(self.codec_stream):     # ordered between the codec parts of two ticks
            self.codec._reset_row(slot)
        if s.voice is not None:       # maya3/engine.py:488-491: the prefix KV, then the prompt after it
            self.backbone.load_prefix_store(slot, s.voice.store, s.voice.length)
        if self.guards is not None:
            self.guards.bind(slot, s.cap, s.suspend)

    def _release(self, s: Seat):
        """maya3/engine.py:632-635."""
        self.backbone.free(s.slot)
        self.free.append(s.slot)

    def cancel(self, s: Seat) -> bool:
        """End a request between ticks (Request.cancel, maya3/engine.py:105-106, acted on at the next tick): a
        waiting request leaves the queue, a decoding one its slot, released at once -- a pipelined tick still in
        flight that carries it runs on and its frame for it is dropped, and the slot's next bind is stream-ordered
        behind that tick.  Returns False when the request had already finished."""
        if s.stop is not None:
            return False
        s.stop = "cancelled"
        if any(p is s for p in self.pending):
            self.pending = [p for p in self.pending if p is not s]
        else:
            self.active = [a for a in self.active if a is not s]
            self._release(s)
        self.stats["cancelled"] = self.stats.get("cancelled", 0) + 1
        return True

    def _admit(self, device=True):
        """maya3/engine.py:449-510 without prompt building: pending requests enter free slots while the tick's row
        budget allows their inline prefill.  A prompt longer than the whole budget is admitted first in its tick:
        its head is prefilled eagerly (chunked backbone steps, the reference's fallback prefill) and its tail rides
        the tick inline.  device=False only claims the slots (the caller resets them later, in stream order, with
        reset_slot) and admits inline prompts only."""
        new, rows = [], len(self.active)
        cap = admission_cap(len(self.active), self.cfg)
        while self.pending and self.free and len(new) < cap:
            s = self.pending[0]
            budget = min(self.max_rows - rows, self.cfg.max_inline_rows)
            if len(s.prompt) > budget:
                if new or not device or budget < 1:
                    break  # admit next tick
                self.pending.pop(0)
                self._bind(s)
                self._prefill_head(s, len(s.prompt) - budget)
            else:
                self.pending.pop(0)
                self._bind(s) if device else self._claim(s)
                s.inline = s.prompt
            new.append(s)
            rows += len(s.inline)
            self.stats["admitted"] += 1
        return new

    @torch.inference_mode()
    def _prefill_head(self, s: Seat, head: int):
        """Prefill the first `head` prompt tokens of a bound seat with eager backbone steps of at most
        max_inline_rows rows; the rest of the prompt becomes its inline part."""
        x = self.embed[torch.from_numpy(s.prompt[:head]).to(self.device)]
        step = self.cfg.max_inline_rows
        for c0 in range(0, head, step):
            self.backbone.step_mixed([], None, [(s.slot, x[c0:c0 + step])])
        s.inline = s.prompt[head:]
        self.stats["eager_prefill_rows"] += head

    # ---------------------------------------------------------------- plan
    def make_plan(self, dec: list, new: list) -> TickPlan:
        """Host plan of one tick (layout of m3_tick_run, plan_layout): decode rows in seat order, then each new seat's
        inline rows; the tick's outputs follow the plan's order.  The backbone step orders the attention's rows
        longest first on the device, so the host does not sort them."""
        p, rb, sb, cb, keys = plan_layout([s.slot for s in dec], [(s.slot, s.inline) for s in new],
                                          self.backbone.lengths_cpu, self.row_buckets, self.buckets,
                                          self.ctx_buckets, self.cfg.max_seats)
        return TickPlan(p, rb, sb, cb, list(dec), list(new), keys)

    def commit(self, tp: TickPlan):
        """Host mirror of what the tick did to the slots' lengths."""
        lc = self.backbone.lengths_cpu
        for s in tp.dec:
            lc[s.slot] += 1
        for s in tp.new:
            lc[s.slot] += len(s.inline)
            self.stats["prefill_rows"] += len(s.inline)

    # ---------------------------------------------------------------- graphs
    def graph_for(self, rb, sb, cb) -> _Graph:
        key = (rb, sb, cb) + self.cb0.flags()   # the penalty / top-p switches are arguments baked into a capture
        g = self.graphs.get(key)
        if g is not None:
            return g
        g = _Graph()
        n = 4 * rb + 2 * sb
        dummy = self.cfg.max_seats
        with torch.inference_mode():
            idle = np.zeros(n, np.int64)
            idle[:rb] = dummy
            idle[3 * rb:4 * rb] = -1
            idle[4 * rb:4 * rb + sb] = dummy
            g.plan = torch.from_numpy(idle).to(self.device)
        g.staging = torch.zeros(n, dtype=torch.long).pin_memory()
        g.evt = None
        g.graph = None
        if self.cfg.use_graphs:
            stream = torch.cuda.Stream()
            stream.wait_stream(torch.cuda.current_stream())
            with torch.cuda.stream(stream):     # an all-padding plan touches only the dummy slot
                for _ in range(2):
                    self._launch(g, rb, sb, cb, stream)
            torch.cuda.current_stream().wait_stream(stream)
            if self.pool is None:
                self.pool = torch.cuda.graph_pool_handle()
            g.graph = torch.cuda.CUDAGraph()
            before = L.load().m3_launch_count()
            with torch.cuda.graph(g.graph, pool=self.pool):
                self._launch(g, rb, sb, cb)
            g.launches = L.load().m3_launch_count() - before   # this library's kernels in one replay
            g.graph.replay()    # the first replay uploads the graph: pay it here, on the idle plan, not in a tick
        else:
            g.launches = None
        self.graphs[key] = g
        return g

    def _launch(self, g, rb, sb, cb, stream=None):
        rep, top_p = self.cb0.flags()
        L.check(L.load().m3_tick_run_main(self._handle, g.plan.data_ptr(), rb, sb, cb, rep, top_p,
                                          L.stream_ptr(stream)), "m3_tick_run_main")

    def codec_for(self, sb, k, beside=True) -> _Codec:
        """The codec part for seat bucket `sb` reading input set `k`; its warm-up and capture decode only the dummy
        slot (the set is staged from an all-padding plan first).  beside: the part runs beside the next tick's main
        part (pipelined ticks), within the codec's SM budget; else alone (a synchronous tick), on every SM."""
        key = (sb, k, beside)
        cg = self.codec_graphs.get(key)
        if cg is not None:
            return cg
        cg = _Codec()
        cg.beside = beside
        lib = L.load()
        with torch.inference_mode():
            cg.packed = torch.zeros(sb, 2 + self.spf // 4, dtype=torch.long, device=self.device)
            idle = torch.full((2 * sb,), self.cfg.max_seats, dtype=torch.long, device=self.device)
            idle[sb:] = 0
        cg.graph = None
        side = torch.cuda.Stream(device=self.device)
        side.wait_stream(torch.cuda.current_stream())
        side.wait_stream(self.codec_stream)
        with torch.cuda.stream(side):
            L.check(lib.m3_tick_stage_codec(self._handle, idle.data_ptr(), 0, sb, k, L.stream_ptr(side)),
                    "m3_tick_stage_codec")
            for _ in range(2 if self.cfg.use_graphs else 0):
                self._launch_codec(cg, sb, k, side)
        torch.cuda.current_stream().wait_stream(side)
        self.codec_stream.wait_stream(side)
        if self.cfg.use_graphs:
            if self.pool is None:
                self.pool = torch.cuda.graph_pool_handle()
            cg.graph = torch.cuda.CUDAGraph()
            before = lib.m3_launch_count()
            with torch.cuda.graph(cg.graph, pool=self.pool):
                self._launch_codec(cg, sb, k)
            cg.launches = lib.m3_launch_count() - before
            with torch.cuda.stream(self.codec_stream):
                cg.graph.replay()   # upload; the set still holds the idle staging
        else:
            cg.launches = None
        self.codec_graphs[key] = cg
        return cg

    def _launch_codec(self, cg, sb, k, stream=None):
        self.codec.set_sm_budget(self._codec_sms if cg.beside else 0)     # read when the kernels are launched
        L.check(L.load().m3_tick_run_codec(self._handle, sb, k, cg.packed.data_ptr(), L.stream_ptr(stream)),
                "m3_tick_run_codec")

    def replay_tick(self, g, tp, k=None, beside=True):
        """Enqueue one planned tick whose plan is already in g.plan: the main part on the current stream, then the
        hand-off of its outputs into codec input set k (after the codec part that last read that set), then the
        codec part on the codec stream (beside: within the codec's SM budget, for a part that runs beside the next
        tick's main part).  Returns the codec part's record."""
        A, B = torch.cuda.current_stream(self.device), self.codec_stream
        if k is None:
            k = self._set
            self._set ^= 1
        cg = self.codec_for(tp.seats, k, beside)
        if g.graph is not None:
            g.graph.replay()
        else:
            self._launch(g, tp.rows, tp.seats, tp.ctx)
        if self._set_free[k] is not None:
            A.wait_event(self._set_free[k])
        L.check(L.load().m3_tick_stage_codec(self._handle, g.plan.data_ptr(), tp.rows, tp.seats, k,
                                             L.stream_ptr(A)), "m3_tick_stage_codec")
        staged = torch.cuda.Event()
        staged.record(A)
        B.wait_event(staged)
        with torch.cuda.stream(B):
            if cg.graph is not None:
                cg.graph.replay()
            else:
                self._launch_codec(cg, tp.seats, k)
        done = torch.cuda.Event()
        done.record(B)
        self._set_free[k] = done
        return cg

    def launches_per_tick(self, g, tp):
        """This library's kernels one tick launches (main graph + hand-off + codec graph), None without graphs."""
        cg = self.codec_graphs.get((tp.seats, 0, True)) or self.codec_graphs.get((tp.seats, 0, False))
        if g.launches is None or cg is None or cg.launches is None:
            return None
        return g.launches + 1 + cg.launches

    # ---------------------------------------------------------------- tick
    def _launch_tick(self, dec, new, beside):
        """Plan one tick, copy its plan host->device, enqueue its main and codec parts (replay_tick) and the
        device->host copy of its packed readout into the next pinned buffer, on the codec stream; the host mirror of
        the KV lengths moves at once.  Returns the tick's (plan, host rows, event recorded after the readout copy)."""
        tp = self.make_plan(dec, new)
        g = self.graph_for(tp.rows, tp.seats, tp.ctx)
        k = self._set
        self._set ^= 1
        self.codec_for(tp.seats, k, beside)     # captured before this tick's plan lands in g.plan
        if g.evt is not None:
            g.evt.synchronize()     # the pinned staging row may still feed the previous copy
        g.staging.numpy()[:] = tp.plan
        g.plan.copy_(g.staging, non_blocking=True)
        g.evt = torch.cuda.Event()
        g.evt.record()
        cg = self.replay_tick(g, tp, k, beside)
        n = len(dec) + len(new)
        host = self._hosts[self._flip][:n]
        self._flip ^= 1
        with torch.cuda.stream(self.codec_stream):
            host.copy_(cg.packed[:n], non_blocking=True)
            evt = torch.cuda.Event()
            evt.record()
        self.commit(tp)
        return tp, host, evt

    @torch.inference_mode()
    def tick(self):
        """One engine tick through the public path: admit, copy the plan host->device, replay, read the packed
        (stop code, cb0, PCM) rows back with one device->host copy and one sync (maya3/engine.py:557-563).
        Returns [(seat, stop code, cb0, int16 PCM or None)] for the seats that ran; the PCM views stay valid until
        the second tick after this one."""
        if self._inflight is not None:
            raise RuntimeError("a pipelined tick is in flight: flush() it before a synchronous tick")
        new = self._admit()
        dec = list(self.active)
        if not dec and not new:
            return []
        tp, host, evt = self._launch_tick(dec, new, beside=False)
        evt.synchronize()
        self._readout = host.numpy()
        return self._deliver(tp.dec + tp.new, self._readout)

    @torch.inference_mode()
    def tick_pipelined(self):
        """The engine loop two ticks deep: launch tick t+1, then read back and deliver tick t, so the host's planning
        and delivery overlap the device's work instead of standing between ticks (the reference's loop,
        maya3/engine.py:514-630, waits on each tick's readout before planning the next).

        Tick t+1 carries every seat of tick t except those tick t is known to finish (its frame exhausts their
        budget); their slots are released before the plan, so admissions refill them in tick t+1 as the synchronous
        loop does.  A seat that tick t's stop code or guard verdict finishes has also run in tick t+1: that frame is
        dropped, and its slot takes admissions from tick t+2 on.  Per seat the frames delivered are the ones
        tick() delivers, one call later.  Returns tick t's [(seat, stop code, cb0, int16 PCM or None)] (empty on the
        first call); flush() delivers the tick still in flight."""
        prev, self._inflight = self._inflight, None
        if prev is not None:
            carried = []
            for s in prev[0].dec + prev[0].new:
                if s.stop is not None:
                    continue                    # finished by an earlier readout: ran speculatively in tick t
                if s.frames + 1 >= s.max_frames:
                    self._release(s)            # every outcome of tick t finishes it; stream order keeps the
                    self._early.add(id(s))      # slot's reset for a new seat behind tick t
                else:
                    carried.append(s)
            self.active = carried
        new = self._admit()
        if self.active or new:
            self._inflight = self._launch_tick(list(self.active), new, beside=True)
        out = self._deliver_inflight(prev) if prev is not None else []
        if self._inflight is not None:
            tp = self._inflight[0]
            self.active = [s for s in tp.dec + tp.new if s.stop is None]
        return out

    @torch.inference_mode()
    def flush(self):
        """Deliver the pipelined tick in flight, if any, without launching another; afterwards tick() may run."""
        prev, self._inflight = self._inflight, None
        return self._deliver_inflight(prev) if prev is not None else []

    def _deliver_inflight(self, rec):
        """Wait for a launched tick's readout and deliver it to the seats still live (a seat finished by the
        readout of the tick before ran in this one speculatively; its row is dropped)."""
        tp, host, evt = rec
        evt.synchronize()
        seats = tp.dec + tp.new
        hv = host.numpy()
        live = [i for i, s in enumerate(seats) if s.stop is None]
        if len(live) < len(seats):
            hv = hv[live]
            seats = [seats[i] for i in live]
        self._readout = hv
        return self._deliver(seats, hv)

    def last_readout(self):
        """The packed readout rows of the last tick delivered, one per seat it delivered, in its order: int64
        [stop | guard verdict << 8 | n_boost << 16, cb0, PCM as int16 pairs...] (a view of pinned host memory)."""
        return self._readout

    @torch.inference_mode()
    def last_outputs(self, n):
        """Copies of the last tick's per-seat device outputs for its first n seats (tick order: decode seats, then
        admitted ones): final-normed backbone hidden [n, hidden] bf16, codes [n, n_q] int64, pre-clamp PCM
        [n, samples_per_frame] fp32."""
        hp, cp, pp = L.vp(), L.vp(), L.vp()
        L.check(L.load().m3_tick_outputs(self._handle, hp, cp, pp), "m3_tick_outputs")
        D, nq = self.geom.backbone.hidden, self.geom.depth.n_q

        def view(ptr, shape, typestr):
            class _Dev:
                __cuda_array_interface__ = {"shape": shape, "typestr": typestr, "data": (int(ptr.value), False),
                                            "version": 3, "strides": None}
            return torch.as_tensor(_Dev(), device=self.device).clone()

        h = view(hp, (n, D), "<i2").view(torch.bfloat16)
        return h, view(cp, (n, nq), "<i8"), view(pp, (n, self.spf), "<f4")

    def deliver_forced(self, seats):
        """Host bookkeeping of a tick whose readout is not read (stops disabled): every seat got one frame."""
        return self._deliver(seats, None)

    def _cap_reason(self, s: Seat) -> str:
        """maya3/engine.py:587-592: the caller's frame budget, the duration prior's cap, or the plain cap."""
        if s.frames >= s.max_frames:
            return "max_frames"
        return "cap_guard" if self.guards.cfg.enabled and s.cap < s.loose_cap else "cap"

    def _deliver(self, seats, hv):
        """Host bookkeeping after a tick: stop codes, frame counts, finished seats; with a readout, the per-seat
        (seat, stop code, cb0, int16 PCM view) tuples.  The readout columns are converted once for all seats."""
        n = len(seats)
        out, finished = [], []
        stops = self.cfg.stops
        if hv is None:
            for s in seats:
                s.new = False
                s.frames += 1
                if s.frames >= s.max_frames:
                    s.stop = "max_frames"
                    finished.append(s)
            frames = n
        else:
            stop_a, verdict_a, boost_a = split_code(hv[:n, 0])
            stop_c = stop_a.tolist()
            cb0s = hv[:n, 1].tolist()
            pcm = list(hv[:n, 2:].view(np.int16))
            guarded = self.guards is not None
            if guarded:
                for s, b in zip(seats, boost_a.tolist()):
                    s.n_boost = b
            verdict_c = verdict_a.tolist() if guarded and stops else None
            if not (stops and stop_a.any()) and verdict_c is None:   # no stop codes: every seat gets its frame
                out = list(zip(seats, stop_c, cb0s, pcm))
                for s in seats:
                    s.new = False
                    s.frames += 1
                    if s.frames >= s.max_frames:
                        s.stop = "max_frames"
                        finished.append(s)
                frames = n
            else:
                frames = 0
                for i, s in enumerate(seats):
                    s.new = False
                    code = stop_c[i]
                    if stops and code:
                        s.stop = REASONS.get(code, str(code))
                        finished.append(s)
                        out.append((s, code, cb0s[i], None))
                        continue
                    s.frames += 1
                    frames += 1
                    out.append((s, code, cb0s[i], pcm[i]))
                    v = verdict_c[i] if verdict_c is not None else 0
                    if v:       # the frame is delivered, then the seat finishes (maya3/engine.py:586-614)
                        s.stop = self._cap_reason(s) if v == 1 else VERDICTS.get(v, str(v))
                        finished.append(s)
                    elif s.frames >= s.max_frames:
                        s.stop = "max_frames"
                        finished.append(s)
        self.stats["frames"] += frames
        self.active = list(seats)
        if finished:
            gone = {id(s) for s in finished}
            for s in finished:
                if id(s) in self._early:
                    self._early.discard(id(s))      # its slot was released when the next tick was planned
                else:
                    self._release(s)
                self.stats["completed"] += 1
            self.active = [s for s in self.active if id(s) not in gone]
        self.stats["ticks"] += 1
        return out


__all__ = ["TickEngine", "TickConfig", "TickPlan", "Seat", "Voice", "FRAME", "FROM_FEEDBACK", "SAMPLING_KEYS",
           "admission_cap", "check_sampling", "frame_budget", "plan_layout"]
