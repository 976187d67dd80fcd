#!/usr/bin/env python
"""Headline benchmark: Maya3 decode ticks under continuous batching at 256 streams per GPU.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl native|reference]

One step = one engine tick over all seats of a replica: backbone decode (+ inline prefill rows of refilled seats),
cb0 sampling, the depth RVQ loop, the Mimi frame and the packed readout.  Seats run prompts of U[64,512] random token
ids for U[100,1500] frames (stops disabled: forced lengths) and are refilled the tick they finish; the replica starts
in the steady state of that process (per-seat KV lengths drawn from its stationary, length-biased distribution), so
KV positions are staggered up to 2011.  Weights are random-init at the benchmark geometry (no checkpoint exists).

Numbers (one JSON line on rank 0):
  value       audio-seconds per second over all GPUs, device-timed: the K ticks' plans are staged in HBM before the
              timed region and replayed back to back (CUDA events on the tick stream, max over ranks);
  e2e         the same metric through the engine's public loop, wall-clocked: per tick the plan is copied
              host->device and the packed (stop, cb0, PCM) readout device->host, with one sync.  The headline runs
              TickEngine.tick_pipelined (tick t+1 launched before tick t is read and delivered); `synchronous` beside
              it runs TickEngine.tick (one tick at a time, as the reference's Engine._tick);
  roofline    the split-KV decode attention (the dominant kernel) re-timed on the live cache after the run;
  reference_gpu the reference's own serving engine (its Engine._tick over its Triton + CUDA-graph StaticBackbone,
              FastDepth and StaticMimi, installed in baseline/_ref) on the same GPU, same seat mix, wall-clocked;
  cpu_baseline the reference's own eager CPU path (fp32) on this host's cores, on a bounded sample (decode ticks of
              8 seats at the same KV-length distribution); `--impl reference` prints that arm's own line.
The KV cache (~60 GB per replica) is far larger than L2, so consecutive ticks never hit in L2 on the cache.
Multi-GPU: one process per GPU, each an independent replica with its own 256 seats (weak scaling, no collective on
the path; torch.distributed only for the start/stop barriers and the max-over-ranks reduction).
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import threading
import time

import numpy as np

REPO = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, REPO)

FRAME_S = 0.08
PROMPT = (64, 512)
TARGET = (100, 1500)
METRIC = "audio-s/s at 256 streams per GPU (continuous batching)"
# DRAM bytes / algorithmic bytes of attn_mma_kernel from an Nsight Compute capture at 256 seats x 1 layer (890.9 MB
# read + written for 877.7 MB of K/V, q and o): the whole-block granularity of the last 16 positions of each row.
ATTN_TRAFFIC_RATIO = 1.0150


def args_():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--impl", default="native", choices=("native", "reference"))
    ap.add_argument("--seats", type=int, default=256)
    ap.add_argument("--capacity", type=int, default=2048)
    ap.add_argument("--seed", type=int, default=0)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-reference-gpu", action="store_true",
                    help="skip the reference engine's run on this GPU (baseline/_ref)")
    ap.add_argument("--no-extra", action="store_true", help="skip the configs[4] box, configs[1] TTFA and configs[3] Mimi runs")
    ap.add_argument("--tick-breakdown", action="store_true",
                    help="time each tick of the device-resident run and print the mean for ticks with and without "
                         "admissions (inline prefill rows), then exit")
    ap.add_argument("--stages", action="store_true",
                    help="print the device time of each stage of a decode tick (backbone, cb0, depth, Mimi) at the "
                         "configs[2] steady state, each stage called through its own mirror object, and exit")
    ap.add_argument("--profile-ticks", type=int, default=0,
                    help="after warm-up, run this many decode-only ticks inside cudaProfilerStart/Stop (for ncu "
                         "--profile-from-start off) and exit")
    return ap.parse_args()


# ------------------------------------------------------------------------------------------------ workload
class Workload:
    """The closed-loop request stream of configs[2]: a finished seat is refilled immediately."""

    def __init__(self, vocab, seed, prompt=PROMPT):
        self.rng = np.random.default_rng(seed)
        self.vocab = vocab
        self.prompt = prompt

    def request(self):
        P = int(self.rng.integers(self.prompt[0], self.prompt[1] + 1))
        T = int(self.rng.integers(TARGET[0], TARGET[1] + 1))
        return self.rng.integers(0, self.vocab, P), T

    def steady_state(self):
        """A seat observed at a random time: its request's length is length-biased (density ~ T), its age uniform."""
        P = int(self.rng.integers(self.prompt[0], self.prompt[1] + 1))
        lo, hi = TARGET
        T = int(np.sqrt(self.rng.uniform(lo * lo, hi * hi)))
        age = int(self.rng.integers(0, T))
        return P, T, age


def init_steady_state(eng, wl, n_seats):
    """Fill every seat with a request part-way through its frames; caches hold synthetic values."""
    import torch
    g = eng.geom
    with torch.inference_mode():
        for k, v in zip(eng.backbone.k, eng.backbone.v):
            k.normal_()
            v.normal_()
        eng.codec.kv.normal_()
        ring = g.mimi.ring
        for _ in range(n_seats):
            P, T, age = wl.steady_state()
            s = eng.submit(wl.rng.integers(0, wl.vocab, P), T)
            eng.pending.remove(s)
            eng._bind(s)
            L = P + age
            eng.backbone.lengths[s.slot] = L
            eng.backbone.lengths_cpu[s.slot] = L
            s.frames = age
            s.new = False
            eng.cb0.frames_t[s.slot] = age
            eng.cb0.ctr_t[s.slot] = age
            eng.cb0.hist_t[s.slot] = torch.from_numpy(wl.rng.integers(0, 2048, eng.cfg.cb0_rep_win))
            eng.depth.row_ctr[s.slot] = age
            tok = 2 * age
            pos = np.arange(max(0, tok - ring), tok)
            kp = np.full(ring, -(1 << 40), np.int64)
            kp[pos % ring] = pos
            with torch.cuda.stream(eng.codec_stream):    # after the slot's codec reset, which runs on that stream
                eng.codec.tokens[s.slot] = tok
                eng.codec.key_pos[s.slot] = torch.from_numpy(kp)
            eng.active.append(s)
    torch.cuda.synchronize()


def top_up(eng, wl):
    while len(eng.pending) < 8:
        p, T = wl.request()
        eng.submit(p, T)


# ------------------------------------------------------------------------------------------------ clocks
class Clocks:
    """nvidia-smi sampling during the timed region (SM clock, max clock, throttle reasons)."""
    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,clocks_event_reasons.hw_slowdown,"
         "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
         "clocks_event_reasons.sw_power_cap")

    def __init__(self, index):
        self.index = index
        self.f = tempfile.NamedTemporaryFile("w+", suffix=".csv", delete=False)
        self.p = None

    def __enter__(self):
        try:
            self.p = subprocess.Popen(["nvidia-smi", "-i", str(self.index), f"--query-gpu={self.Q}",
                                       "--format=csv,noheader,nounits", "-lms", "200"], stdout=self.f,
                                      stderr=subprocess.DEVNULL)
        except OSError:
            self.p = None
        time.sleep(0.3)
        return self

    def __exit__(self, *a):
        if self.p is not None:
            self.p.terminate()
            try:
                self.p.wait(5)
            except subprocess.TimeoutExpired:
                self.p.kill()

    def summary(self):
        self.f.flush()
        rows = []
        for line in open(self.f.name):
            parts = [x.strip() for x in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                rows.append((float(parts[1]), float(parts[2]), float(parts[3]), parts[5:9]))
            except ValueError:
                continue
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unavailable"]}
        busy = [r for r in rows if r[2] > 250] or rows
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in busy for i, v in enumerate(r[3]) if v.lower() == "active"})
        return {"sm_mhz": statistics.median(r[0] for r in busy), "sm_max_mhz": max(r[1] for r in rows),
                "reasons": reasons, "samples": len(busy)}


# ------------------------------------------------------------------------------------------------ native arm
def run_native(a, rank, world, local):
    import torch
    import torch.distributed as dist

    from maya2_native_b200 import weights as WG
    from maya2_native_b200.config import BASELINE
    from maya2_native_b200.engine import TickConfig, TickEngine

    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    g = BASELINE
    W = WG.generate(WG.all_shapes(g), seed=a.seed, device=dev)
    cfg = TickConfig(max_seats=a.seats, capacity=a.capacity, stops=False, max_inline_rows=512)
    eng = TickEngine(g, W, cfg, device=dev)
    del W
    wl = Workload(g.backbone.vocab, a.seed * 7919 + rank)
    init_steady_state(eng, wl, a.seats)
    top_up(eng, wl)
    for _ in range(a.warmup):
        eng.tick()
        top_up(eng, wl)
    if a.profile_ticks:
        # decode-only ticks, the common kind (the queue is held back, so nothing is admitted), with their graph
        # captured by an untimed tick before the profiled region
        held, eng.pending = eng.pending, []
        eng.tick()
        torch.cuda.synchronize()
        torch.cuda.cudart().cudaProfilerStart()
        for _ in range(a.profile_ticks):
            eng.tick()
        torch.cuda.synchronize()
        torch.cuda.cudart().cudaProfilerStop()
        eng.pending = held
        return {"profiled_ticks": a.profile_ticks, "kind": "decode-only"}

    # ---- device-resident run: plan K ticks on the host, stage them in HBM, replay back to back
    plans = []
    for _ in range(a.steps):
        new = eng._admit(device=False)
        dec = list(eng.active)
        tp = eng.make_plan(dec, new)
        eng.commit(tp)
        eng.deliver_forced(tp.dec + tp.new)
        top_up(eng, wl)
        plans.append(tp)
    for tp in plans:
        eng.graph_for(tp.rows, tp.seats, tp.ctx)
        for k in (0, 1):
            eng.codec_for(tp.seats, k)
    staged = torch.from_numpy(np.concatenate([tp.plan for tp in plans])).to(dev)
    offs = np.cumsum([0] + [len(tp.plan) for tp in plans])
    frames = sum(len(tp.dec) + len(tp.new) for tp in plans)
    stream = torch.cuda.current_stream()
    ev = [torch.cuda.Event(enable_timing=True) for _ in range(len(plans) + 1)]
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    from maya2_native_b200 import _lib as L
    lib = L.load()
    launches = 0
    with Clocks(local) as clk:
        c0 = lib.m3_launch_count()
        ev[0].record(stream)
        for k, tp in enumerate(plans):
            for s in tp.new:
                eng.reset_slot(s)
            gr = eng.graph_for(tp.rows, tp.seats, tp.ctx)
            gr.plan.copy_(staged[offs[k]:offs[k + 1]], non_blocking=True)
            cg = eng.replay_tick(gr, tp)      # main part here, codec part on the codec stream beside the next tick
            launches += gr.launches + cg.launches
            ev[k + 1].record(stream)
        stream.wait_stream(eng.codec_stream)  # the window ends with the last tick's codec part
        ev_end = torch.cuda.Event(enable_timing=True)
        ev_end.record(stream)
        torch.cuda.synchronize()
        launches += lib.m3_launch_count() - c0          # eager launches in the region (slot resets)
    dev_ms = ev[0].elapsed_time(ev_end)
    tick_ms = [ev[k].elapsed_time(ev[k + 1]) for k in range(len(plans))]
    if a.tick_breakdown:
        adm = [k for k, tp in enumerate(plans) if tp.new]
        dec = [k for k, tp in enumerate(plans) if not tp.new]
        eng.close()
        return {"ticks": len(plans), "decode_only": {"n": len(dec), "mean_ms": float(np.mean([tick_ms[k] for k in dec]))},
                "with_admission": {"n": len(adm), "mean_ms": float(np.mean([tick_ms[k] for k in adm])) if adm else None,
                                   "rows": [int(plans[k].rows) for k in adm],
                                   "prefill_rows": [int(sum(len(s.prompt) for s in plans[k].new)) for k in adm],
                                   "ms": [round(tick_ms[k], 3) for k in adm]}}
    status = eng.device_status()

    # ---- end to end through the public tick: H2D plan + D2H readout + sync every tick, wall clock.  The graphs of
    # the buckets these ticks can reach (any admission rows at the full seat bucket, the two largest context buckets)
    # are captured first and W public ticks run untimed, so no graph is captured inside the timed window.
    for cb in eng.ctx_buckets[-2:]:
        for rb in (r for r in eng.row_buckets if r >= eng.buckets[-1]):
            eng.graph_for(rb, eng.buckets[-1], cb)
    for k in (0, 1):
        for beside in (False, True):     # the synchronous and the pipelined loop
            eng.codec_for(eng.buckets[-1], k, beside)
    def public_run(pipelined):
        """K ticks through the public loop, wall-clocked: tick() (plan, launch, read back, deliver, one tick at a
        time) or tick_pipelined() (tick t+1 launched before tick t is read; the pipeline starts empty and the last
        tick is flushed inside the window, so the window holds exactly K launched and delivered ticks)."""
        step = eng.tick_pipelined if pipelined else eng.tick
        for _ in range(a.warmup):
            step()
            top_up(eng, wl)
        if pipelined:
            eng.flush()
        n_graphs = len(eng.graphs) + len(eng.codec_graphs)
        adm0, rows0 = eng.stats["admitted"], eng.stats["prefill_rows"]
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
        frames_out = 0
        t0 = time.perf_counter()
        for _ in range(a.steps):
            out = step()
            frames_out += len(out)
            top_up(eng, wl)
        if pipelined:
            frames_out += len(eng.flush())
        torch.cuda.synchronize()
        mix = {"admitted": eng.stats["admitted"] - adm0, "prefill_rows": eng.stats["prefill_rows"] - rows0,
               "graphs_captured_in_window": len(eng.graphs) + len(eng.codec_graphs) - n_graphs}
        return time.perf_counter() - t0, frames_out, mix

    row_bytes = (2 + eng.spf // 4) * 8                    # one packed readout row copied back per frame
    sync_s, sync_frames, sync_mix = public_run(False)
    e2e_s, e2e_frames, e2e_mix = public_run(True)
    d2h = e2e_frames * row_bytes
    h2d = int(np.mean([len(tp.plan) * 8 for tp in plans]))   # the tick plan (slots, offsets, prompt token ids)

    # ---- roofline of the decode attention on the live cache (the last tick's rows)
    tp = eng.make_plan(list(eng.active), [])
    gr = eng.graph_for(tp.rows, tp.seats, tp.ctx)
    gr.plan.copy_(torch.from_numpy(tp.plan).to(dev))
    eng.replay_tick(gr, tp)     # leaves this step's q / slots / positions in the scratch
    eng.commit(tp)
    eng.deliver_forced(tp.dec)
    bg = g.backbone
    reps = 20
    torch.cuda.synchronize()
    a0, a1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a0.record(stream)
    for i in range(reps):
        L.check(lib.m3_backbone_attention(eng.backbone._handle, i % bg.layers, tp.rows, tp.ctx, L.stream_ptr()))
    a1.record(stream)
    torch.cuda.synchronize()
    attn_ms = a0.elapsed_time(a1) / reps
    kv_bytes = tp.keys * bg.kv_heads * bg.head_dim * 2 * 2
    qo_bytes = tp.rows * bg.heads * bg.head_dim * 2 * 2
    attn_bytes = kv_bytes + qo_bytes

    # ---- reduce over ranks
    clocks = clk.summary()
    dev_ms, e2e_ms, frames, e2e_frames = reduce_over_ranks(dev_ms, e2e_s * 1e3, frames, e2e_frames, world, dev)
    _, sync_ms, _, sync_frames = reduce_over_ranks(0.0, sync_s * 1e3, 0, sync_frames, world, dev)
    value = frames * FRAME_S / (dev_ms / 1e3)
    e2e = e2e_frames * FRAME_S / (e2e_ms / 1e3)
    e2e_sync = sync_frames * FRAME_S / (sync_ms / 1e3)
    peaks = {}
    try:
        peaks = json.load(open(os.path.join(REPO, "MEASURED_PEAKS.json")))
    except OSError:
        pass
    hbm = peaks.get("hbm_gbs")
    peak_src = "measured" if hbm else "fallback"
    hbm = hbm or 6650.0
    achieved = attn_bytes / (attn_ms / 1e3) / 1e9
    line = {
        "metric": METRIC, "value": round(value, 2), "unit": "audio-s/s", "n_gpus": world, "steps": a.steps,
        "warmup": a.warmup, "ms_per_step": round(dev_ms / a.steps, 4), "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "bf16", "data": "synthetic (random-init weights, random prompt token ids)",
        "config": {"workload": "configs[2]: continuous batching, 256 seats/GPU, prompts U[64,512], targets "
                               "U[100,1500] frames, refill on finish, KV positions staggered up to 2011",
                   "seats_per_gpu": a.seats, "capacity": a.capacity, "geometry": "Qwen3-0.6B backbone, 4x1024 depth "
                   "(8 codebooks), Mimi 8 codebooks", "parallelism": f"replicas x{world}",
                   "l2": "inputs larger than L2 (KV cache ~60 GB per replica)"},
        "e2e": {"value": round(e2e, 2), "unit": "audio-s/s", "h2d_bytes_per_step": h2d,
                "d2h_bytes_per_step": int(d2h / max(a.steps, 1)), **e2e_mix,
                "loop": "TickEngine.tick_pipelined (tick t+1 launched before tick t is read)",
                "synchronous": {"value": round(e2e_sync, 2), "loop": "TickEngine.tick (one tick at a time, as the "
                                "reference's Engine._tick)", **sync_mix},
                "note": "each loop runs its own K ticks of the live workload after the device-timed ones; admissions "
                        "(inline prefill rows) make a tick slower, so the windows differ by their mix"},
        "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": hbm, "unit": "GB/s",
                     "frac": round(achieved / hbm, 4), "traffic": int(attn_bytes * ATTN_TRAFFIC_RATIO),
                     "traffic_source": "ncu DRAM bytes of the same kernel at 256 seats x 1 layer, scaled by keys",
                     "kernel": "attn_mma_kernel (split-KV decode attention, splits merged in the launch)",
                     "peak_source": peak_src, "algorithmic_bytes": int(attn_bytes), "launch_ms": round(attn_ms, 5),
                     "note": "the peak is a copy benchmark (read + write); this kernel only reads, so it can pass 1.0"},
        "tick_ms": round(dev_ms / a.steps, 4),
        "tick_ms_p50": round(float(np.percentile(tick_ms, 50)), 4),
        "tick_ms_p99": round(float(np.percentile(tick_ms, 99)), 4),
        "frames_timed": int(frames), "device_status": status,
        "value_window": {"admitted": int(sum(len(tp.new) for tp in plans)),
                         "prefill_rows": int(sum(len(s.inline) for tp in plans for s in tp.new))},
        "clocks": clocks,
        "gpu_launches": int(launches),
    }
    if not a.no_extra:
        line["box"] = run_box(eng, a, rank, world, dev, value / world)
    eng.close()
    del eng
    torch.cuda.empty_cache()
    if world == 1 and not a.no_extra:
        line["ttfa"] = run_ttfa(dev, a.seed)
        line["mimi"] = run_mimi(dev, a.seed)
    return line


BOX_PROMPT = (20, 400)
BOX_LOAD = 0.9


def run_box(eng, a, rank, world, dev, cap_per_gpu, duration=12.0, warm=10.0):
    """open-loop Poisson arrivals at 90% of the measured capacity (cap_per_gpu audio-s/s per replica,
    from the configs[2] run just before), routed round-robin over the `world` replicas (maya2_native_b200.router),
    prompts of U[20,400] random token ids, frame budgets U[100,1500].  Each replica starts EMPTY and runs its engine
    loop against the wall clock: before every tick it submits the arrivals whose time has come.  The first `warm`
    seconds (about two request lifetimes) bring the seats to the load's own steady state; the next `duration`
    seconds are measured.  Reported: frames delivered inside the window (any stream) / the window, and TTFA over
    EVERY stream that arrived inside the window -- arrival -> the end of the TickEngine.tick that returns its first
    PCM frame (queueing for a free seat included); a stream still without audio when the window closes counts with
    its wait so far (a lower bound), so slow streams are not dropped from the percentiles."""
    import torch
    import torch.distributed as dist

    from maya2_native_b200.router import poisson_arrivals, requests, share
    mean_frames = (TARGET[0] + TARGET[1]) / 2
    lam = BOX_LOAD * cap_per_gpu / (mean_frames * FRAME_S)          # streams per second per replica
    arr = poisson_arrivals(lam * world, warm + duration, seed=a.seed + 4)
    mine = requests(arr, eng.geom.backbone.vocab, indices=share(len(arr), rank, world), prompt=BOX_PROMPT,
                    frames=TARGET, seed=a.seed + 4)
    for s in list(eng.active):
        eng._release(s)
    eng.active, eng.pending = [], []
    # graphs of the buckets this load reaches (every seat bucket from empty to full, any admission rows, the two
    # largest context buckets), captured before the clock starts
    tc = time.perf_counter()
    for cb in eng.ctx_buckets[-2:]:
        for sb in eng.buckets:
            for rb in (r for r in eng.row_buckets if r >= sb):
                eng.graph_for(rb, sb, cb)
    for sb in eng.buckets:
        for k in (0, 1):
            eng.codec_for(sb, k, beside=False)     # the box runs the synchronous loop
    torch.cuda.synchronize()
    print(f"box: rank {rank} captured {len(eng.graphs)} graphs in {time.perf_counter() - tc:.2f} s", file=sys.stderr)
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    t0 = time.perf_counter()
    k, arrived, ttfa, frames, occ = 0, {}, [], 0, []
    t_start = None
    n_graphs = len(eng.graphs) + len(eng.codec_graphs)
    while True:
        now = time.perf_counter() - t0
        if now >= warm + duration:
            break
        if t_start is None and now >= warm:
            t_start, frames, occ, n_graphs = now, 0, [], len(eng.graphs) + len(eng.codec_graphs)
        while k < len(mine) and mine[k].t <= now:
            r = mine[k]
            s = eng.submit(r.prompt, r.frames)
            arrived[id(s)] = (r.t, s)
            k += 1
        out = eng.tick()
        t = time.perf_counter() - t0
        occ.append(len(out))
        for s, _, _, pcm in out:
            if pcm is not None:
                frames += 1
                ta = arrived.pop(id(s), None)
                if ta is not None and ta[0] >= warm:
                    ttfa.append((t - ta[0]) * 1e3)
    torch.cuda.synchronize()
    t_end = time.perf_counter() - t0
    window = t_end - t_start
    waiting = [(t_end - ta) * 1e3 for ta, _ in arrived.values() if ta >= warm]   # no audio yet: wait so far
    if len(eng.graphs) + len(eng.codec_graphs) > n_graphs:
        print(f"box: rank {rank} captured {len(eng.graphs) + len(eng.codec_graphs) - n_graphs} graphs in the window: "
              f"{list(eng.graphs)[-3:]}", file=sys.stderr)
    local = (ttfa + waiting, frames, window, float(np.mean(occ)) if occ else 0.0, len(waiting), len(mine),
             len(eng.graphs) + len(eng.codec_graphs) - n_graphs)
    return summarize_box(local, world, a.seats, cap_per_gpu)


def summarize_box(local, world, seats, cap_per_gpu):
    """Combine the replicas' configs[4] results (every rank passes its own; all ranks get the summary): local =
    (TTFA ms list over the window's arrivals, frames delivered in the window, window s, mean busy seats, window
    arrivals still without audio at its end, arrivals routed here, graphs captured inside the window)."""
    if world > 1:
        import torch.distributed as dist
        got = [None] * world
        dist.all_gather_object(got, local)
    else:
        got = [local]
    all_ttfa = [x for g in got for x in g[0]]
    agg = sum(g[1] for g in got) * FRAME_S / max(g[2] for g in got)
    return {"workload": f"configs[4]: Poisson arrivals at {BOX_LOAD:.0%} of the measured capacity, routed "
                        f"round-robin over {world} replicas ({seats} seats each), prompts U[20,400] ids, targets "
                        "U[100,1500] frames",
            "audio_s_per_s": round(agg, 1), "offered_audio_s_per_s": round(BOX_LOAD * cap_per_gpu * world, 1),
            "ttfa_p50_ms": round(float(np.percentile(all_ttfa, 50)), 2) if all_ttfa else None,
            "ttfa_p99_ms": round(float(np.percentile(all_ttfa, 99)), 2) if all_ttfa else None,
            "window_arrivals": len(all_ttfa), "arrivals": int(sum(g[5] for g in got)),
            "mean_busy_seats_per_gpu": round(float(np.mean([g[3] for g in got])), 1),
            "without_audio_at_end": int(sum(g[4] for g in got)), "window_s": round(max(g[2] for g in got), 3),
            "graphs_captured_in_window": int(sum(g[6] for g in got)),
            "measured": "replicas start empty, 10 s warm-up under the load, then a 12 s window; audio-s/s = frames "
                        "delivered in the window; TTFA over every arrival in the window: arrival -> end of the "
                        "TickEngine.tick returning its first PCM frame, or the wait so far at the window's end"}


def reduce_over_ranks(dev_ms, e2e_ms, frames, e2e_frames, world, device):
    """Max of the timed durations and sum of the frames over ranks (every rank is one replica)."""
    if world == 1:
        return dev_ms, e2e_ms, frames, e2e_frames
    import torch
    import torch.distributed as dist
    t = torch.tensor([dev_ms, e2e_ms], device=device, dtype=torch.float64)
    n = torch.tensor([float(frames), float(e2e_frames)], device=device, dtype=torch.float64)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    dist.all_reduce(n, op=dist.ReduceOp.SUM)
    return float(t[0]), float(t[1]), float(n[0]), float(n[1])


def run_ttfa(dev, seed, n_req=100, warm=8):
    """B = 1, capacity 1024, one prompt of 300 uniform-random token ids per request (generator seed i),
    temperature 0.8 / top-k 50 for cb0 and depth.  TTFA = submit -> the tick that returns the request's first PCM
    frame (inline prefill of the prompt + the first frame), host clock; the engine is warm (graphs captured)."""
    import torch

    from maya2_native_b200 import weights as WG
    from maya2_native_b200.config import BASELINE
    from maya2_native_b200.engine import TickConfig, TickEngine
    W = WG.generate(WG.all_shapes(BASELINE), seed=seed, device=dev)
    cfg = TickConfig(max_seats=1, capacity=1024, temp=0.8, top_k=50, cb0_temp=0.8, cb0_top_k=50, stops=False)
    eng = TickEngine(BASELINE, W, cfg, device=dev)
    del W
    out = []
    for i in range(warm + n_req):
        prompt = np.random.default_rng(i).integers(0, BASELINE.backbone.vocab, 300)
        t0 = time.perf_counter()
        s = eng.submit(prompt, 2)
        first = None
        for _ in range(8):
            res = eng.tick()
            if first is None and any(x[0] is s and x[3] is not None for x in res):
                first = time.perf_counter()
            if s.stop is not None:
                break
        if first is None:
            raise RuntimeError("TTFA request produced no audio")
        if i >= warm:
            out.append((first - t0) * 1e3)
    eng.close()
    del eng
    torch.cuda.empty_cache()
    return {"p50_ms": round(float(np.percentile(out, 50)), 3), "p99_ms": round(float(np.percentile(out, 99)), 3),
            "n": n_req, "workload": "configs[1]: B=1, capacity 1024, 300-token prompts, temp 0.8 / top-k 50",
            "measured": "submit -> first PCM frame out of TickEngine.tick (host clock, warm engine)"}


def run_mimi(dev, seed, streams=256, warm=130, frames=50):
    """StaticMimi.decode over 256 streams, codes U[0, 2048) x 8 codebooks (seed 0), after 130 warm
    frames (the 250-position window and the 256-entry ring are full); device-timed with CUDA events.  hbm_gbs =
    (ring K/V read + decoder weights) per frame batch / time."""
    import torch

    from maya2_native_b200 import weights as WG
    from maya2_native_b200.codec import StaticMimi
    from maya2_native_b200.config import BASELINE
    g = BASELINE.mimi
    shapes = {k: v for k, v in WG.all_shapes(BASELINE).items() if k.startswith("mimi.")}
    W = WG.generate(shapes, seed=seed, device=dev)
    codec = StaticMimi(W, streams, batch_buckets=(streams,), geom=g, device=dev)
    wbytes = sum(int(np.prod(v)) for v in shapes.values()) * 2
    del W
    gen = torch.Generator(device=dev).manual_seed(0)
    codes = torch.randint(0, g.codebook_size, (warm + frames, streams, g.n_q), device=dev, generator=gen)
    slots = torch.arange(streams, device=dev)
    with torch.inference_mode():
        for f in range(warm):
            codec.decode(slots, codes[f])
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for f in range(warm, warm + frames):
            codec.decode(slots, codes[f])
        e1.record()
        torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / frames
    kv = streams * g.layers * 2 * g.heads * g.ring * (g.hidden // g.heads) * 2
    # the fused SEANet stages' transposed convs alone (m3_mimi_convt re-runs one on the buffers the last frame left)
    import ctypes

    from maya2_native_b200 import _lib as L
    lib, convt = L.load(), []
    for st in range(len(g.ratios)):
        nb = ctypes.c_int64(0)
        if lib.m3_mimi_convt(codec._handle, st, streams, ctypes.byref(nb), L.stream_ptr()) != 0:
            continue                                        # not a fused stage
        c0, c1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        c0.record()
        for _ in range(20):
            L.check(lib.m3_mimi_convt(codec._handle, st, streams, ctypes.byref(nb), L.stream_ptr()))
        c1.record()
        torch.cuda.synchronize()
        us = c0.elapsed_time(c1) / 20 * 1e3
        convt.append({"stage": st, "us": round(us, 2), "bytes": int(nb.value),
                      "hbm_gbs": round(nb.value / (us / 1e6) / 1e9, 1)})
    codec.close()
    return {"samples_per_s": round(streams * g.samples_per_frame / (ms / 1e3)),
            "ms_per_frame": round(ms, 4), "hbm_gbs": round((kv + wbytes) / (ms / 1e3) / 1e9, 1),
            "convt": convt,
            "workload": "configs[3]: 256 streams, codes U[0,2048) x 8, 130 warm frames, StaticMimi.decode; convt = "
                        "each fused transposed-conv stage alone (bf16 input read + output written, bytes / time)"}


def run_stages(a):
    """Per-stage device time of a decode tick: every seat decodes one frame, stage by stage through the mirror
    objects (StaticBackbone.step, the cb0 sampler, FastDepth, StaticMimi.decode), CUDA events between the stages."""
    import torch

    from maya2_native_b200 import weights as WG
    from maya2_native_b200.config import BASELINE
    from maya2_native_b200.engine import TickConfig, TickEngine
    dev = torch.device("cuda", 0)
    g = BASELINE
    W = WG.generate(WG.all_shapes(g), seed=a.seed, device=dev)
    eng = TickEngine(g, W, TickConfig(max_seats=a.seats, capacity=a.capacity, stops=False), device=dev)
    del W
    wl = Workload(g.backbone.vocab, a.seed * 7919)
    init_steady_state(eng, wl, a.seats)
    slots = [s.slot for s in eng.active]
    idx = torch.tensor(slots, device=dev)
    names = ("backbone", "cb0", "depth", "mimi")
    times = {k: [] for k in names}
    with torch.inference_mode():
        for it in range(a.warmup + a.steps):
            ev = [torch.cuda.Event(enable_timing=True) for _ in range(5)]
            x = eng.feedback[idx]
            ev[0].record()
            h = eng.backbone.step(slots, x)
            ev[1].record()
            _, cb0 = eng.cb0(h, idx)
            ev[2].record()
            codes, fb = eng.depth(slots, h, cb0)
            ev[3].record()
            eng.codec.decode(idx, codes)
            ev[4].record()
            eng.feedback[idx] = fb
            torch.cuda.synchronize()
            if it >= a.warmup:
                for k, n in enumerate(names):
                    times[n].append(ev[k].elapsed_time(ev[k + 1]))
    med = {n: round(float(np.median(v)), 4) for n, v in times.items()}
    eng.close()
    return {"stages_ms": med, "sum_ms": round(sum(med.values()), 4), "seats": a.seats, "steps": a.steps,
            "note": "eager stage calls (backbone not graph-captured), events between stages"}


# ------------------------------------------------------------------------------------------------ CPU arm
def cpu_tick_sample(seats, seed=0, reps=1):
    """The fp32 CPU oracle (numpy port of the reference's eager path) on `seats` seats at the configs[2] KV-length
    distribution; returns (seconds per tick, threads)."""
    from maya2_native_b200 import weights as WG
    from maya2_native_b200.config import BASELINE
    from oracle.tick import OracleTick
    g = BASELINE
    shapes = {k: v for k, v in WG.all_shapes(g).items() if "embed_tokens" not in k}
    W = {k: v.numpy() for k, v in WG.generate(shapes, seed=seed).items()}
    wl = Workload(g.backbone.vocab, seed)
    cap = 2048
    o = OracleTick(W, g, seats, cap, "fp32")
    bg = g.backbone
    block = np.random.default_rng(seed).standard_normal((bg.kv_heads, 256, bg.head_dim)).astype(np.float32)
    for s in range(seats):
        P, T, age = wl.steady_state()
        n = P + age
        reps_ = -(-n // 256)
        kv = np.tile(block, (1, reps_, 1))[:, :n]
        o.bb.k[:, s, :, :n] = kv[None]
        o.bb.v[:, s, :, :n] = kv[None]
        o.bb.lengths[s] = n
    times = []
    for _ in range(reps):
        t0 = time.perf_counter()
        o.tick(list(range(seats)))
        times.append(time.perf_counter() - t0)
    return min(times), os.cpu_count()


REF_CPU_SEATS = 8


def run_reference(a, rank, world):
    """--impl reference: the reference's own eager CPU path (baseline/_ref: StaticBackbone 'gather', Engine._cb0,
    FastDepth._compute, StaticMimi._forward, fp32) on this host's cores, one step = one decode tick of 8 seats at the
    configs[2] KV-length distribution, W untimed ticks then K timed ones.  Without the install, the numpy oracle
    port of the same path stands in (kind "port")."""
    from baseline import reference_arm as RA
    from maya2_native_b200.config import BASELINE
    seats = REF_CPU_SEATS
    why = RA.unavailable()
    if why is None:
        wl = Workload(BASELINE.backbone.vocab, a.seed * 7919)
        times, cores = RA.cpu_tick(BASELINE, wl, seats, a.capacity, ticks=max(1, a.steps), warmup=a.warmup,
                                   seed=a.seed)
        config0 = RA.cpu_config0(BASELINE, seed=a.seed)
        kind = "reference"
        sample = (f"one decode tick of {seats} seats at the configs[2] KV-length distribution through the "
                  "reference's own eager CPU path (fp32)")
    else:
        times, cores = [], os.cpu_count()
        for _ in range(max(1, a.steps)):
            sec, cores = cpu_tick_sample(seats, a.seed, reps=1)
            times.append(sec)
        kind = "port"
        config0 = None
        sample = f"one decode tick of {seats} seats at the configs[2] KV-length distribution, fp32 numpy port ({why})"
    sec = float(np.mean(times))
    v = seats * FRAME_S / sec
    extra = {"configs0": config0} if config0 else {}
    return {**extra, "metric": METRIC, "value": round(v, 4), "unit": "audio-s/s", "n_gpus": world, "steps": len(times),
            "warmup": a.warmup if kind == "reference" else 0, "ms_per_step": round(sec * 1e3, 2),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "impl": "reference",
            "config": {"workload": f"configs[2] seat mix, CPU sample: decode ticks of {seats} seats", "seats": seats,
                       "capacity": a.capacity},
            "cpu_baseline": {"value": round(v, 4), "unit": "audio-s/s", "cores": cores, "kind": kind,
                             "sample": sample},
            "e2e": {"value": round(v, 4), "unit": "audio-s/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}


def reference_cpu_line(a):
    """The --impl reference line for a short CPU sample (2 timed ticks after 1 warm), run in a child process: the
    reference's CPU path runs its Triton sampler in the interpreter, a process-wide switch."""
    env = {k: v for k, v in os.environ.items() if k not in ("RANK", "WORLD_SIZE", "LOCAL_RANK", "MASTER_ADDR",
                                                            "MASTER_PORT", "LOCAL_WORLD_SIZE")}
    env["CUDA_VISIBLE_DEVICES"] = ""
    cmd = [sys.executable, os.path.join(REPO, "bench.py"), "--impl", "reference", "--steps", "2", "--warmup", "1",
           "--capacity", str(a.capacity), "--seed", str(a.seed)]
    r = subprocess.run(cmd, capture_output=True, text=True, env=env, timeout=900)
    for line in r.stdout.splitlines()[::-1]:
        if line.startswith("{"):
            return json.loads(line)
    raise RuntimeError(f"reference CPU sample failed (rc {r.returncode}): {r.stderr[-400:]}")


def run_reference_gpu(a, dev, line):
    """The reference's own serving engine (Triton + CUDA graphs, baseline/_ref) on this GPU at configs[2] -- same seat
    mix, steady-state start, W untimed and K timed ticks -- at bf16 and at its default dtypes, plus its configs[1]
    TTFA; reported beside the native arm's numbers."""
    from baseline import reference_arm as RA
    from maya2_native_b200.config import BASELINE
    why = RA.unavailable()
    if why is not None:
        return {"unavailable": why}
    wl = Workload(BASELINE.backbone.vocab, a.seed * 7919)
    out = RA.gpu_arm(dev, wl, a.seats, a.capacity, steps=a.steps, warmup=a.warmup, seed=a.seed)
    out["native_e2e_over_reference"] = round(line["e2e"]["value"] / out["value"], 3)
    out["native_value_over_reference"] = round(line["value"] / out["value"], 3)
    if "ttfa" in line and "ttfa" in out:
        out["ttfa"]["reference_p50_over_native"] = round(out["ttfa"]["p50_ms"] / line["ttfa"]["p50_ms"], 3)
    return out


def main():
    a = args_()
    rank = int(os.environ.get("RANK", 0))
    world = int(os.environ.get("WORLD_SIZE", 1))
    local = int(os.environ.get("LOCAL_RANK", 0))
    if a.stages:
        print(json.dumps(run_stages(a)), flush=True)
        return
    if a.impl == "reference":
        if rank == 0:
            print(json.dumps(run_reference(a, rank, world)), flush=True)
        return
    import torch
    import torch.distributed as dist
    if world > 1:
        import datetime
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=600), device_id=torch.device("cuda", local))
    with torch.inference_mode():
        line = run_native(a, rank, world, local)
    if rank == 0 and world == 1 and not a.no_extra and not a.no_reference_gpu and "e2e" in line:
        try:
            line["reference_gpu"] = run_reference_gpu(a, torch.device("cuda", local), line)
        except Exception as exc:                      # reported, not fatal: the native line still stands
            line["reference_gpu"] = {"unavailable": f"{type(exc).__name__}: {exc}"[:300]}
    if rank == 0 and world == 1 and not a.no_cpu_baseline:
        ref = reference_cpu_line(a)
        line["cpu_baseline"] = ref["cpu_baseline"]
    if rank == 0:
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
