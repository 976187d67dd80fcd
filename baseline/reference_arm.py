"""The reference's own decode tick, run unmodified from an install of the reference in ``baseline/_ref``.

``bench.py`` measures this library against two arms built from the reference's code itself:

* ``gpu_arm`` -- the reference's serving engine on the same B200: its ``Engine._build_fast`` constructs its own
  ``StaticBackbone(attention='triton', fuse_rope=True)``, ``FastDepth(fused=True)`` and ``StaticMimi`` with their
  CUDA graphs, and its own ``Engine._tick`` runs the ticks (admission with inline prefill or the eager HF fallback,
  the graphed backbone step, ``_cb0``, the depth graph, the Mimi graph, the int16 pack and the one device->host
  readout with its sync, then delivery).  Only ``Engine._plan`` -- text normalisation, prompt packing and voices,
  which sit above the decode path -- is replaced: a request here is a prompt of random backbone token ids whose
  embedding is the backbone's own ``embed_text``, with a frame budget and no minimum-frame stop (forced lengths).
* ``cpu_tick`` -- the reference's eager CPU path: ``StaticBackbone._forward`` with ``attention='gather'``,
  ``Engine._cb0``, ``FastDepth._compute`` and ``StaticMimi._forward`` in fp32 on the host cores.

The install is ``python -m pip install --no-index --no-build-isolation --no-deps --find-links /opt/wheelhouse
--target baseline/_ref <reference checkout>`` (``--no-deps``: the reference pins torch 2.8.0 / transformers 5.6.2,
which the offline wheelhouse does not hold; the image's torch and transformers are used).  ``baseline/_ref`` is not
part of this repository's history; it travels with the working tree to the machine that runs the benchmark.

Weights are this package's seeded random-init tensors (``maya2_native_b200.weights``) loaded under the reference's
own state-dict names, at the benchmark geometry; the reference's hard-coded depth geometry
(tts/model/depth_v2.py:45-48, serve/fast_depth.py:26-29) is patched to it before its modules are built.
"""
from __future__ import annotations

import collections
import os
import sys
import threading
import time
import types

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
REF = os.path.join(HERE, "_ref")
FRAME_S = 0.08
NO_STOP = 1 << 30          # minimum frames before a controlled stop may fire: never (forced lengths)


def unavailable():
    """None when the reference install is present, else the reason it is not."""
    for part in ("serve/fast_backbone.py", "serve/fast_depth.py", "serve/fast_codec.py", "maya3/engine.py"):
        if not os.path.exists(os.path.join(REF, part)):
            return f"reference install missing ({os.path.join('baseline/_ref', part)} not found)"
    return None


def use_reference():
    """Put the reference install on sys.path (raises when it is absent)."""
    why = unavailable()
    if why:
        raise RuntimeError(why)
    if REF not in sys.path:
        sys.path.insert(0, REF)


_use_reference = use_reference


def _patch_depth(g):
    """Set the reference's depth-geometry module constants (tts/model/depth_v2.py:45-48, serve/fast_depth.py:26-29)."""
    import serve.fast_depth as FD
    import tts.model.depth_v2 as DV
    gol = list(g.group_of_level)
    for mod in (DV, FD):
        mod.D, mod.H, mod.LAYERS, mod.GROUP_OF_LEVEL = g.d, g.heads, g.layers, gol
    DV.FFN, DV.RANK, DV.N_GROUPS = g.ffn, g.rank, g.n_groups
    FD.HEAD, FD.N_LEVELS = g.d // g.heads, g.n_q


def _load_named(module, prefix, seed, device):
    """Fill a reference module's parameters and buffers from the seeded generator, by state-dict name."""
    from maya2_native_b200 import weights as WG
    gen = "cuda" if str(device).startswith("cuda") else None
    sd = module.state_dict()
    new = {k: WG.make(prefix + k, v.shape, seed, device=gen).to(device=device, dtype=v.dtype)
           for k, v in sd.items() if k != "lm_head.weight"}
    module.load_state_dict(new, strict=False)   # lm_head is tied to the embedding


def build_models(geom, device, seed=0, mimi_dtype=None):
    """The reference's model objects at `geom` on `device`: a ``tts.model.backbone.Backbone`` (bf16 on a GPU, fp32 on
    the CPU) around an HF ``Qwen3ForCausalLM``, ``DepthV2`` in fp32 (the engine's ``model.depth.float()``), the
    backbone-width ``AudioInputEmbed`` and an HF ``MimiModel``.  Returns (model namespace, mimi)."""
    import torch
    from transformers import MimiConfig, MimiModel, Qwen3Config, Qwen3ForCausalLM
    from transformers.models.qwen3.modeling_qwen3 import Qwen3RotaryEmbedding

    _use_reference()
    from tts.model.backbone import Backbone

    gpu = str(device).startswith("cuda")
    dt = torch.bfloat16 if gpu else torch.float32
    b = geom.backbone
    cfg = Qwen3Config(hidden_size=b.hidden, num_hidden_layers=b.layers, num_attention_heads=b.heads,
                      num_key_value_heads=b.kv_heads, head_dim=b.head_dim, intermediate_size=b.ffn,
                      vocab_size=b.vocab, rms_norm_eps=b.eps, tie_word_embeddings=True,
                      rope_parameters={"rope_theta": b.rope_theta, "rope_type": "default"})
    with torch.device("meta"):
        lm = Qwen3ForCausalLM(cfg)
    lm = lm.to_empty(device=device)
    lm.model.rotary_emb = Qwen3RotaryEmbedding(cfg, device=device)   # non-persistent buffers: rebuilt, not loaded
    _load_named(lm, "", seed, device)
    lm.tie_weights()
    lm = lm.to(dt).eval()
    bb = Backbone.__new__(Backbone)            # the reference wrapper without its tokenizer download
    torch.nn.Module.__init__(bb)
    bb.lm = lm
    bb.d_model = b.hidden
    bb.cb0_head = torch.nn.Linear(b.hidden, b.n_cb0, bias=False, device=device)
    _load_named(bb.cb0_head, "cb0_head.", seed, device)
    bb.cb0_head.to(dt)

    depth, audio_in = build_depth(geom, device, seed, dt)

    m = geom.mimi
    mcfg = MimiConfig(hidden_size=m.hidden, num_quantizers=m.n_q, num_semantic_quantizers=m.n_semantic,
                      codebook_size=m.codebook_size, codebook_dim=m.codebook_dim,
                      vector_quantization_hidden_dimension=m.codebook_dim, num_hidden_layers=m.layers,
                      num_attention_heads=m.heads, num_key_value_heads=m.heads, intermediate_size=m.ffn,
                      sliding_window=m.window, upsampling_ratios=list(m.ratios), num_filters=m.num_filters,
                      upsample_groups=m.hidden, sampling_rate=int(12.5 * m.samples_per_frame), frame_rate=12.5,
                      rope_parameters={"rope_theta": m.rope_theta, "rope_type": "default"})
    with torch.device(device):
        mimi = MimiModel(mcfg)
    _load_named(mimi, "mimi.", seed, device)
    for mod in mimi.modules():
        if hasattr(mod, "_embed"):
            mod._embed = None                    # codebook cache rebuilt from the loaded embed_sum
    mimi = mimi.to(mimi_dtype or dt).eval()
    model = types.SimpleNamespace(backbone=bb.eval(), depth=depth, audio_in=audio_in)
    return model, mimi


def build_depth(geom, device, seed=0, audio_dtype=None):
    """The reference's ``DepthV2`` (fp32, as the engine keeps it: maya3/engine.py:158) and backbone-width
    ``AudioInputEmbed`` at `geom` on `device`, from the seeded weights.  Returns (depth, audio_in)."""
    import torch
    _use_reference()
    _patch_depth(geom.depth)
    from tts.model.audio_io import AudioInputEmbed
    from tts.model.depth_v2 import DepthV2
    d = geom.depth
    with torch.device("meta"):
        depth = DepthV2(d_backbone=d.d_backbone, n_q=d.n_q, n_codes=d.n_codes)
    depth = depth.to_empty(device=device)
    _load_named(depth, "depth.", seed, device)
    depth = depth.float().eval()
    audio_in = AudioInputEmbed(d.d_backbone, n_q=d.n_q, n_codes=d.n_codes).to(device)
    _load_named(audio_in, "audio_in.", seed, device)
    audio_in = audio_in.to(audio_dtype or (torch.bfloat16 if str(device).startswith("cuda") else torch.float32))
    return depth, audio_in.eval()


# ------------------------------------------------------------------------------------------------ GPU arm
def engine(model, mimi, device, seats, capacity, depth_dtype, build=None, **cfg):
    """A reference ``Engine`` built by its own ``_build_fast`` (or by `build(engine)` in its place) around the given
    models (``Engine.__init__`` would load a checkpoint, a tokenizer and a voice registry, none of which the decode
    path uses).  The fp32 depth stack is kept after FastDepth copies it (``free_reference_depth=False``) so further
    engines can be built from the same models; it is not read by the tick."""
    import torch
    from maya3 import engine as ME
    from maya3 import guards as G
    torch.backends.cuda.enable_cudnn_sdp(False)          # maya3/engine.py:153-154
    torch.backends.cuda.matmul.allow_tf32 = False
    E = ME.Engine.__new__(ME.Engine)
    E.cfg = ME.EngineConfig(max_seats=seats, capacity=capacity, depth_dtype=depth_dtype,
                            guards=G.GuardConfig(enabled=False), free_reference_depth=False, **cfg)
    E.device = device
    E.log = lambda *a, **k: None
    E.model = model
    E.mimi = mimi
    if build is None:
        E._build_fast()
    else:
        build(E)
    E._pending = collections.deque()
    E._calls = collections.deque()
    E._cv = threading.Condition()
    E._stop = False
    E._thread = None
    E.stats = {"ticks": 0, "admitted": 0, "completed": 0, "prefix_hits": 0, "prefix_misses": 0,
               "fallback_prefill": 0}
    E.tick_ms = collections.deque(maxlen=20000)
    E.phase_ms = {}
    E.failed = None
    E.warm = True

    def plan(req):
        """Stand-in for Engine._plan (maya3/engine.py:394-418): the prompt is the backbone embedding of the request's
        token ids; cap = its frame budget; no controlled stop (forced lengths); no suspend windows."""
        ids = torch.as_tensor(req.ids, device=device, dtype=torch.long)
        prompt = model.backbone.embed_text(ids)[None].to(torch.bfloat16)
        return prompt, int(len(req.ids)), int(req.target), int(req.target), NO_STOP, ()
    E._plan = plan
    return E


def voice(model, device):
    """A plain voice (no prefix, null speaker memory): the fields Engine._admit/_bind read."""
    import torch
    return types.SimpleNamespace(ts=0, kv=None, builder=None,
                                 mem=model.depth.spk_memory(torch.zeros(1, 1, 192, device=device), "ecapa",
                                                            null_mask=torch.tensor([True], device=device)),
                                 rmask=torch.ones(1, 1, dtype=torch.bool, device=device))


def _tick_run(model, mimi, device, wl, seats, capacity, steps, warmup, depth_dtype):
    """configs[2] through one reference engine: steady-state start, W untimed ticks, K ticks wall-clocked."""
    import torch
    from maya3 import engine as ME
    t_build = time.perf_counter()
    with torch.inference_mode():
        E = engine(model, mimi, device, seats, capacity, depth_dtype)
        vc = voice(model, device)
    delivered = [0]

    def on_event(kind, payload):
        if kind == "audio":
            delivered[0] += 1

    def request(ids, frames):
        r = ME.Request(["-"], "en", vc, on_event)
        r.ids, r.target = ids, frames
        return r

    def top_up():
        while len(E._pending) < 8:
            p, T = wl.request()
            E._pending.append(request(p, T))

    # steady state of the renewal process, as the native arm starts (bench.init_steady_state)
    ring = E.codec.ring
    with torch.inference_mode():
        for k, v in zip(E.backbone.k, E.backbone.v):
            k.normal_()
            v.normal_()
        E.codec.kv.normal_()
        for _ in range(seats):
            P, T, age = wl.steady_state()
            seat = E._bind(request(wl.rng.integers(0, wl.vocab, P), T), T, T, NO_STOP, ())
            s, L = seat.slot, P + age
            E.backbone.lengths[s] = L
            E.backbone.lengths_cpu[s] = L
            seat.frames = age
            seat.new = False
            E.frames_t[s] = age
            E.ctr_t[s] = age
            E.hist_t[s] = torch.from_numpy(wl.rng.integers(0, 2048, E.cfg.cb0_rep_win))
            E.depth.row_ctr[s] = age
            tok = 2 * age
            E.codec.tokens[s] = tok
            pos = np.arange(max(0, tok - ring), tok)
            kp = np.full(ring, -(1 << 40), np.int64)
            kp[pos % ring] = pos
            E.codec.key_pos[s] = torch.from_numpy(kp)
            E.active.append(seat)
        top_up()
        # graphs of the buckets a full replica reaches (decode rows + inline prefill rows up to the row budget, the
        # two largest context buckets, the top seat buckets), captured before the clock starts
        big = [b for b in E.row_buckets if b >= E.buckets[-1]]
        E.backbone.warmup(batch_buckets=big, ctx_buckets=E.backbone.ctx_buckets[-2:])
        near = [b for b in E.buckets if b >= 0.8 * seats]
        E.depth.warmup(near)
        E.codec.warmup(near)
        torch.cuda.synchronize()
    build_s = time.perf_counter() - t_build
    for _ in range(warmup):
        E._tick()
        top_up()

    def n_graphs():
        return len(E.backbone.graphs) + len(E.depth.graphs) + len(E.codec._buckets)
    g0, fb0, f0 = n_graphs(), E.stats["fallback_prefill"], delivered[0]
    admitted0 = E.stats["admitted"]
    per = []
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    for _ in range(steps):
        ts = time.perf_counter()
        E._tick()
        per.append(time.perf_counter() - ts)
        top_up()
    torch.cuda.synchronize()
    wall = time.perf_counter() - t0
    frames = delivered[0] - f0
    out = {"value": round(frames * FRAME_S / wall, 2), "unit": "audio-s/s",
           "tick_ms": round(wall / steps * 1e3, 4),
           "tick_ms_p50": round(float(np.percentile(per, 50)) * 1e3, 4),
           "tick_ms_p99": round(float(np.percentile(per, 99)) * 1e3, 4),
           "steps": steps, "warmup": warmup, "frames": int(frames),
           "admitted": E.stats["admitted"] - admitted0,
           "eager_fallback_prefills": E.stats["fallback_prefill"] - fb0,
           "graphs_captured_in_window": n_graphs() - g0, "build_and_capture_s": round(build_s, 1)}
    del E
    torch.cuda.empty_cache()
    return out


def _ttfa_run(model, mimi, device, vocab, n_req, warm, prompt_len=300, capacity=1024):
    """configs[1] through a one-seat reference engine: a request of `prompt_len` uniform-random token ids (generator
    seed = request index), temperature 0.8 / top-k 50 for cb0 and depth; TTFA = submit -> the reference's first
    'audio' event (maya3/bench/bench_engine.py:49-69 measures to the same callback), host clock, warm engine."""
    import torch
    from maya3 import engine as ME
    with torch.inference_mode():
        E = engine(model, mimi, device, 1, capacity, "bf16", temp=0.8, top_k=50, cb0_temp=0.8, cb0_top_k=50)
        vc = voice(model, device)
    out = []
    for i in range(warm + n_req):
        first = []
        r = ME.Request(["-"], "en", vc, lambda k, p: first.append(time.perf_counter()) if k == "audio" else None)
        r.ids, r.target = np.random.default_rng(i).integers(0, vocab, prompt_len), 2
        t0 = time.perf_counter()
        E._pending.append(r)
        for _ in range(8):
            E._tick()
            if r.done:
                break
        if not first:
            raise RuntimeError("reference TTFA request produced no audio")
        if i >= warm:
            out.append((first[0] - t0) * 1e3)
    del E
    torch.cuda.empty_cache()
    return {"p50_ms": round(float(np.percentile(out, 50)), 3), "p99_ms": round(float(np.percentile(out, 99)), 3),
            "n": n_req, "workload": f"configs[1]: B=1, capacity {capacity}, {prompt_len}-token prompts, temp 0.8 / "
                                    "top-k 50, bf16"}


def gpu_arm(device, wl, seats=256, capacity=2048, steps=50, warmup=10, seed=0, geom=None, ttfa_requests=50):
    """The reference's own engine on one GPU: configs[2] (bench.py's Workload `wl`: the same request stream and
    steady-state start as the native arm) at bf16 throughout and at the engine's default dtypes (depth fp16, Mimi
    fp32: maya3/engine.py:53,165), and configs[1]'s B=1 TTFA.  Returns the measurements as a dict."""
    import copy

    import torch
    from maya2_native_b200.config import BASELINE
    geom = geom or BASELINE
    _use_reference()
    with torch.inference_mode():
        model, mimi32 = build_models(geom, device, seed, mimi_dtype=torch.float32)
        mimi16 = copy.deepcopy(mimi32).to(torch.bfloat16)
    out = _tick_run(model, mimi16, device, wl, seats, capacity, steps, warmup, "bf16")
    out["dtypes"] = {"backbone": "bf16", "depth": "bf16", "mimi": "bf16"}
    out["measured"] = ("wall clock around the reference's own Engine._tick (one D2H + sync per tick), same seat mix "
                       "and steady-state start as the native arm")
    d = _tick_run(model, mimi32, device, wl, seats, capacity, steps, warmup, "fp16")
    d["dtypes"] = {"backbone": "bf16", "depth": "fp16", "mimi": "fp32"}
    out["engine_defaults"] = d
    if ttfa_requests:
        out["ttfa"] = _ttfa_run(model, mimi16, device, geom.backbone.vocab, ttfa_requests, 8)
    del model, mimi16, mimi32
    torch.cuda.empty_cache()
    return out


# ------------------------------------------------------------------------------------------------ CPU arm
_CPU_MODELS = {}


def _cpu_models(geom, seed):
    """The reference's model objects on the CPU in fp32, built once per (geometry, seed) in this process."""
    import torch
    key = (geom, seed)
    if key not in _CPU_MODELS:
        _CPU_MODELS[key] = build_models(geom, torch.device("cpu"), seed)
    return _CPU_MODELS[key]


def _cb0_state(model, seats, top_k=64, rep=0.8):
    """The engine's per-slot sampler tensors (maya3/engine.py:210-223) for `seats` seats on the CPU."""
    import torch
    from maya3 import engine as ME
    m = seats + 1
    return types.SimpleNamespace(
        model=model, cfg=ME.EngineConfig(max_seats=seats, cb0_rep=rep), _any_rep=False, _any_top_p=False,
        temp_t=torch.full((m,), 0.9), topk_t=torch.full((m,), top_k, dtype=torch.long),
        topp_t=torch.ones(m), rep_t=torch.full((m,), rep), aeos_bias=torch.zeros(m),
        seed_t=torch.arange(m, dtype=torch.int32) + 17, ctr_t=torch.zeros(m, dtype=torch.int32),
        hist_t=torch.full((m, 12), -1, dtype=torch.long), frames_t=torch.zeros(m, dtype=torch.long),
        min_t=torch.full((m,), NO_STOP, dtype=torch.long), hazard_t=torch.zeros(m))


def _cpu_setup():
    os.environ["TRITON_INTERPRET"] = "1"        # Engine._cb0's row_exponential is a Triton kernel: run it on the host
    import torch
    use_reference()
    torch.set_num_threads(os.cpu_count())


def cpu_tick(geom, wl, seats, capacity=2048, ticks=2, warmup=1, seed=0):
    """Seconds of each of `ticks` decode ticks (after `warmup` untimed ones) of `seats` seats through the reference's
    eager CPU path in fp32, and the threads used.  KV lengths follow wl's steady state; caches hold noise."""
    _cpu_setup()
    import torch
    from maya3 import engine as ME
    from serve.fast_backbone import StaticBackbone
    from serve.fast_codec import StaticMimi
    from serve.fast_depth import FastDepth
    with torch.inference_mode():
        model, mimi = _cpu_models(geom, seed)
        sb = StaticBackbone(model.backbone, seats, capacity=capacity, ctx_buckets=(capacity,), attention="gather",
                            use_graphs=False)
        fd = FastDepth(model, seats, dtype=torch.float32, batch_buckets=(seats,), seed=seed + 1, fused=False)
        sm = StaticMimi(mimi, seats, batch_buckets=(seats,), ring=geom.mimi.ring)
        mem = model.depth.spk_memory(torch.zeros(1, 1, 192), "ecapa", null_mask=torch.tensor([True]))
        for s in range(seats):
            fd.set_speaker(s, mem, torch.ones(1, 1, dtype=torch.bool))
        gen = torch.Generator().manual_seed(seed)
        for k, v in zip(sb.k, sb.v):
            k.normal_(generator=gen)
            v.normal_(generator=gen)
        lens = [wl.steady_state() for _ in range(seats)]
        for s, (P, T, age) in enumerate(lens):
            sb.lengths[s] = P + age
            sb.lengths_cpu[s] = P + age
        st = _cb0_state(model, seats)
        slots = torch.arange(seats)
        x = torch.randn(seats, geom.backbone.hidden, generator=gen) * 0.02
        times = []
        for it in range(warmup + ticks):
            t0 = time.perf_counter()
            h = sb._forward(slots, x, torch.ones(seats, dtype=torch.long), capacity)
            _, cb0 = ME.Engine._cb0(st, h, slots)
            codes, fb = fd._compute(slots, h, cb0)
            sm._forward(slots, codes[:, :, None])
            times.append(time.perf_counter() - t0)
            x = fb
    return times[warmup:], torch.get_num_threads()


def cpu_config0(geom, frames=50, seats=4, capacity=512, prompt_len=200, seed=0):
    """configs[0] on the reference's eager CPU path in fp32: B = 4 seats, KV capacity 512, prompts
    torch.randint(0, vocab, (4, 200)) from generator seed 0 prefilled by the HF model itself into DynamicCaches
    installed with StaticBackbone.load_slot (the engine's eager fallback, maya3/engine.py:497-507), then `frames`
    greedy frames (cb0 at top-k 1 without penalty, FastDepth greedy) with each frame's feedback fed back
    (maya3/engine.py:544-556).  Returns the timings."""
    _cpu_setup()
    import torch
    from maya3 import engine as ME
    from serve.fast_backbone import StaticBackbone
    from serve.fast_codec import StaticMimi
    from serve.fast_depth import FastDepth
    with torch.inference_mode():
        model, mimi = _cpu_models(geom, seed)
        sb = StaticBackbone(model.backbone, seats, capacity=capacity, ctx_buckets=(capacity,), attention="gather",
                            use_graphs=False)
        fd = FastDepth(model, seats, dtype=torch.float32, batch_buckets=(seats,), seed=seed + 1, greedy=True,
                       fused=False)
        sm = StaticMimi(mimi, seats, batch_buckets=(seats,), ring=geom.mimi.ring)
        mem = model.depth.spk_memory(torch.zeros(1, 1, 192), "ecapa", null_mask=torch.tensor([True]))
        for s in range(seats):
            fd.set_speaker(s, mem, torch.ones(1, 1, dtype=torch.bool))
        st = _cb0_state(model, seats, top_k=1, rep=0.0)
        prompts = torch.randint(0, geom.backbone.vocab, (seats, prompt_len), generator=torch.Generator().manual_seed(0))
        slots = torch.arange(seats)
        t0 = time.perf_counter()
        emb = model.backbone.embed_text(prompts)
        h = torch.empty(seats, geom.backbone.hidden)
        for s in range(seats):
            hs, cache = model.backbone(emb[s:s + 1], use_cache=True)
            sb.load_slot(s, cache, prompt_len)
            h[s] = hs[0, -1]
        t1 = time.perf_counter()
        for f in range(frames):
            if f:
                h = sb._forward(slots, fb, torch.ones(seats, dtype=torch.long), capacity)
            _, cb0 = ME.Engine._cb0(st, h, slots)
            codes, fb = fd._compute(slots, h, cb0)
            sm._forward(slots, codes[:, :, None])
        t2 = time.perf_counter()
    dec = t2 - t1
    return {"seats": seats, "frames": frames, "prefill_s": round(t1 - t0, 3), "s_per_frame": round(dec / frames, 4),
            "audio_s_per_s": round(seats * frames * FRAME_S / dec, 4), "cores": torch.get_num_threads(),
            "workload": f"configs[0]: B={seats}, capacity {capacity}, {prompt_len}-token prompts (HF eager prefill "
                        f"-> load_slot), {frames} greedy frames with feedback, fp32, the reference's own eager CPU path"}
