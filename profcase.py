"""Small GPU cases for Nsight Compute captures: a few GB on the device, inputs still far larger than L2.

    python profcase.py attention [--seats 64] [--layers 2] [--steps 3]
    python profcase.py tick [--seats 64] [--steps 3]

Part of the measurement harness beside bench.py (the summaries under profiles/ name the command that made them);
not imported by the library.

attention: the backbone step over `seats` decode rows at the configs[2] KV-length distribution (mean ~790 keys),
           benchmark width, `layers` layers (2 layers x 64 seats ~ 1 GB of K/V); run under
           `ncu --clock-control none -k regex:attn_mma -c 3` (every ncu command needs --clock-control none: without
           it ncu locks the GPU's clocks, a setting the GPU's next user would inherit).
tick:      the full engine tick at the benchmark geometry with fewer seats.
mimi:      StaticMimi.decode at the benchmark geometry over `seats` streams.
gaps:      per-node cost of a CUDA graph of dependent tiny kernels.
overlap:   backbone step and Mimi decode (or the depth loop: --with depth) timed back to back and concurrently on
           two streams.
guard:     the loop guard (m3_guard_step) over `seats` seats on due frames, alone and as a graph node.
"""
from __future__ import annotations

import argparse
import dataclasses
import os
import sys

import numpy as np
import torch

sys.path.insert(0, os.path.dirname(os.path.abspath(__file__)))


def _lengths(n, rng):
    P = rng.integers(64, 513, n)
    T = np.sqrt(rng.uniform(100 ** 2, 1500 ** 2, n)).astype(np.int64)
    return P + (rng.random(n) * T).astype(np.int64)


@torch.inference_mode()
def attention(a):
    from maya2_native_b200 import weights as WG
    from maya2_native_b200.backbone import StaticBackbone
    from maya2_native_b200.config import BASELINE
    g = dataclasses.replace(BASELINE.backbone, layers=a.layers)
    dev = torch.device("cuda", 0)
    W = WG.generate({k: v for k, v in WG.backbone_shapes(g).items() if "embed" not in k}, device=dev)
    sb = StaticBackbone(W, a.seats, capacity=2048, batch_buckets=(a.seats,), ctx_buckets=(2048,), use_graphs=False,
                        geom=g, device=dev)
    for k, v in zip(sb.k, sb.v):
        k.normal_()
        v.normal_()
    rng = np.random.default_rng(0)
    L = _lengths(a.seats, rng)
    sb.lengths[:a.seats] = torch.from_numpy(L).to(dev)
    for s, n in enumerate(L):
        sb.lengths_cpu[s] = int(n)
    x = torch.randn(a.seats, g.hidden, device=dev, dtype=torch.bfloat16)
    order = [int(s) for s in np.argsort(-L, kind="stable")]   # longest first, the order the step visits rows in
    for _ in range(a.steps):
        sb.step(order, x)
    torch.cuda.synchronize()
    print(f"attention case: {a.seats} seats, {a.layers} layers, mean keys {L.mean():.0f}")


@torch.inference_mode()
def tick(a):
    from maya2_native_b200 import weights as WG
    from maya2_native_b200.config import BASELINE
    from maya2_native_b200.engine import TickConfig, TickEngine
    dev = torch.device("cuda", 0)
    W = WG.generate(WG.all_shapes(BASELINE), device=dev)
    eng = TickEngine(BASELINE, W, TickConfig(max_seats=a.seats, capacity=2048, stops=False), device=dev)
    rng = np.random.default_rng(0)
    for _ in range(a.seats):
        eng.submit(rng.integers(0, BASELINE.backbone.vocab, int(rng.integers(64, 200))), 1000)
    while eng.pending:
        eng.tick()
    for _ in range(a.steps):
        eng.tick()
    torch.cuda.synchronize()
    print(f"tick case: {a.seats} seats, {a.steps} ticks")


@torch.inference_mode()
def mimi(a):
    """StaticMimi.decode at the benchmark geometry over `seats` streams (codes U[0, 2048)), `steps` frames."""
    from maya2_native_b200 import weights as WG
    from maya2_native_b200.codec import StaticMimi
    from maya2_native_b200.config import BASELINE
    dev = torch.device("cuda", 0)
    g = BASELINE.mimi
    shapes = {k: v for k, v in WG.all_shapes(BASELINE).items() if k.startswith("mimi.")}
    codec = StaticMimi(WG.generate(shapes, device=dev), a.seats, batch_buckets=(a.seats,), geom=g, device=dev)
    gen = torch.Generator(device=dev).manual_seed(0)
    slots = torch.arange(a.seats, device=dev)
    for _ in range(a.steps):
        codec.decode(slots, torch.randint(0, g.codebook_size, (a.seats, g.n_q), device=dev, generator=gen))
    torch.cuda.synchronize()
    print(f"mimi case: {a.seats} streams, {a.steps} frames")


@torch.inference_mode()
def gaps(a):
    """Per-node cost of a CUDA graph of dependent tiny kernels (one-element adds on one stream): the launch and
    dependency overhead that every small kernel of the tick pays."""
    dev = torch.device("cuda", 0)
    x = torch.zeros(1, device=dev)
    for n in (100, 400):
        side = torch.cuda.Stream()
        side.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(side):
            x.add_(1)
        torch.cuda.current_stream().wait_stream(side)
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            for _ in range(n):
                x.add_(1)
        g.replay()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(10):
            g.replay()
        e1.record()
        torch.cuda.synchronize()
        print(f"graph of {n} dependent tiny kernels: {e0.elapsed_time(e1) / 10 / n * 1e3:.3f} us per node")


@torch.inference_mode()
def overlap(a):
    """Could another stage hide under the backbone step?  Graph-captured backbone step (decode rows of `seats` seats,
    configs[2] KV-length distribution, benchmark width, all layers) and, with `--with mimi`, the Mimi decode of
    `seats` streams or, with `--with depth`, the depth loop of `seats` seats, timed back to back on one stream and
    concurrently on two."""
    from maya2_native_b200 import weights as WG
    from maya2_native_b200.backbone import StaticBackbone
    from maya2_native_b200.codec import StaticMimi
    from maya2_native_b200.config import BASELINE
    from maya2_native_b200.depth import FastDepth
    dev = torch.device("cuda", 0)
    g = BASELINE
    W = WG.generate({k: v for k, v in WG.all_shapes(g).items() if k != "model.embed_tokens.weight"}, device=dev)
    sb = StaticBackbone(W, a.seats, capacity=2048, batch_buckets=(a.seats, 512), ctx_buckets=(2048,), use_graphs=True,
                        geom=g.backbone, device=dev)
    if a.with_ in ("depth", "depth+mimi", "prefill+depth", "depth-halves"):
        fd = FastDepth(W, a.seats, batch_buckets=(a.seats,), geom=g.depth, device=dev)
        hd = torch.randn(a.seats, g.depth.d_backbone, device=dev, dtype=torch.bfloat16)
        cb0 = torch.randint(0, 2048, (a.seats,), device=dev)
        dslots = list(range(a.seats))
        other = lambda: fd(dslots, hd, cb0)
    if a.with_ == "depth-halves":
        hs = a.seats // 2
        fa = FastDepth(W, a.seats, batch_buckets=(hs,), geom=g.depth, device=dev)
        fb = FastDepth(W, a.seats, batch_buckets=(hs,), geom=g.depth, device=dev)
        full = other
        first = lambda: fa(dslots[:hs], hd[:hs], cb0[:hs])
        other = lambda: fb(dslots[hs:], hd[hs:], cb0[hs:])
        t_full = None
    if a.with_ == "depth+mimi":
        codec = StaticMimi(W, a.seats, batch_buckets=(a.seats,), geom=g.mimi, device=dev)
        first, other = other, (lambda: codec.decode(idx, codes))
    if a.with_ == "prefill+depth":     # slot `seats - 1` is emptied and refilled with the prompt every call
        xp = torch.randn(a.prompt, g.backbone.hidden, device=dev, dtype=torch.bfloat16)

        def first():
            sb.free(a.seats - 1)
            for c0 in range(0, a.prompt, 512):
                sb.step_mixed([], None, [(a.seats - 1, xp[c0:c0 + 512])])
    elif a.with_ == "mimi":
        codec = StaticMimi(W, a.seats, batch_buckets=(a.seats,), geom=g.mimi, device=dev)
        other = lambda: codec.decode(idx, codes)
    for k, v in zip(sb.k, sb.v):
        k.normal_()
        v.normal_()
    rng = np.random.default_rng(0)
    L = _lengths(a.seats, rng)
    sb.lengths[:a.seats] = torch.from_numpy(L).to(dev)
    for s, n in enumerate(L):
        sb.lengths_cpu[s] = int(n)
    slots = list(range(a.seats))
    x = torch.randn(a.seats, g.backbone.hidden, device=dev, dtype=torch.bfloat16)
    codes = torch.randint(0, 2048, (a.seats, g.mimi.n_q), device=dev)
    idx = torch.arange(a.seats, device=dev)
    if a.with_ not in ("depth+mimi", "prefill+depth", "depth-halves"):
        first = lambda: sb.step(slots, x)
    first()
    other()
    torch.cuda.synchronize()
    s1, s2 = torch.cuda.Stream(), torch.cuda.Stream()

    def run(concurrent, reps=10):
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        torch.cuda.synchronize()
        e0.record()
        cur = torch.cuda.current_stream()
        for _ in range(reps):
            s1.wait_stream(cur)
            s2.wait_stream(cur)
            with torch.cuda.stream(s1):
                first()
            with torch.cuda.stream(s2 if concurrent else s1):
                other()
            cur.wait_stream(s1)
            cur.wait_stream(s2)
        e1.record()
        torch.cuda.synchronize()
        if a.with_ not in ("depth+mimi", "prefill+depth", "depth-halves"):   # the backbone steps advanced lengths
            for s in range(a.seats):
                sb.lengths_cpu[s] -= reps
            sb.lengths[:a.seats] -= reps
        return e0.elapsed_time(e1) / reps

    def alone(fn, reps=10):
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        torch.cuda.synchronize()
        e0.record()
        for _ in range(reps):
            fn()
        e1.record()
        torch.cuda.synchronize()
        return e0.elapsed_time(e1) / reps

    t_bb = alone(first)
    if a.with_ not in ("depth+mimi", "prefill+depth", "depth-halves"):
        sb.lengths[:a.seats] -= 10
        for s in range(a.seats):
            sb.lengths_cpu[s] -= 10
    t_other = alone(other)
    name = {"depth+mimi": "depth", "prefill+depth": f"prefill of {a.prompt}",
            "depth-halves": f"depth of {a.seats // 2}"}.get(a.with_, "backbone step")
    if a.with_ == "depth-halves":
        print(f"depth of all {a.seats} seats on one handle: {alone(full):.3f} ms")
    print(f"seats {a.seats}: {name} {t_bb:.3f} ms, {a.with_.split('+')[-1]} {t_other:.3f} ms, sequential "
          f"{run(False):.3f} ms, concurrent {run(True):.3f} ms")


# (label, M, N, K) of the linear layers of one configs[2] tick
TICK_GEMMS = [("bb.qkv", 256, 4096, 1024), ("bb.o", 256, 1024, 2048), ("bb.gu", 256, 6144, 1024),
              ("bb.down", 256, 1024, 3072), ("bb.qkv+pf", 768, 4096, 1024), ("depth.qkv n8", 2048, 3072, 1024),
              ("depth.o n8", 2048, 1024, 1024), ("depth.f1 n8", 2048, 3072, 1024), ("depth.f2 n8", 2048, 1024, 3072),
              ("depth.qkv n2", 512, 3072, 1024), ("depth.f2 last", 256, 1024, 3072), ("depth.head", 256, 2048, 1024),
              ("mimi.qkv", 512, 1536, 512), ("mimi.fc1", 512, 2048, 512), ("mimi.fc2", 512, 512, 2048),
              ("mimi.conv0", 512, 1024, 3584), ("mimi.convt8", 512, 8192, 1024), ("mimi.res8", 4096, 256, 1536),
              ("mimi.convt6", 4096, 3072, 512), ("mimi.res6", 24576, 128, 768), ("mimi.convt5", 24576, 1280, 256),
              ("mimi.res5", 122880, 64, 384), ("mimi.convt4", 122880, 512, 128), ("mimi.res4", 491520, 32, 192),
              ("mimi.res4k1", 491520, 64, 32)]


@torch.inference_mode()
def gemm(a):
    """Time m3_gemm_bf16 (GEMV for M <= 8, cuBLAS above) on the tick's linear-layer shapes (bf16 out; CUDA events
    over graph replays).  --cold cycles through enough weight copies (> 2x L2) that every launch streams its weights
    from HBM, as the tick's 28 layers do."""
    from maya2_native_b200 import _lib as L
    dev = torch.device("cuda", 0)
    lib = L.load()
    print(f"{'layer':16s} {'M':>7s} {'N':>5s} {'K':>5s}        us     TF/s")
    for name, M, N, K in TICK_GEMMS:
        if a.shape and name != a.shape:
            continue
        x = torch.randn(M, K, device=dev).to(torch.bfloat16)
        copies = max(1, -(-(256 << 20) // (N * K * 2))) if a.cold else 1
        ws = [torch.randn(N, K, device=dev).to(torch.bfloat16) for _ in range(min(copies, 64))]
        y = torch.empty(M, N, device=dev, dtype=torch.bfloat16)
        reps = 64 if a.cold else 20

        def call(i):
            w = ws[i % len(ws)]
            L.check(lib.m3_gemm_bf16(x.data_ptr(), K, w.data_ptr(), K, y.data_ptr(), N, M, N, K, 0, L.stream_ptr()))
        side = torch.cuda.Stream()
        side.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(side):
            for i in range(3):
                call(i)
        torch.cuda.current_stream().wait_stream(side)
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):      # launches replayed without host overhead, as in the tick graph
            for i in range(reps):
                call(i)
        graph.replay()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(5):
            graph.replay()
        e1.record()
        torch.cuda.synchronize()
        us = e0.elapsed_time(e1) / (5 * reps) * 1e3
        print(f"{name:16s} {M:7d} {N:5d} {K:5d}  {us:8.2f} {2 * M * N * K / us / 1e6:8.1f}", flush=True)


@torch.inference_mode()
def guard(a):
    """m3_guard_step over `seats` seats whose histories are full and whose every update is due (frame 100, the loop
    rule evaluated for all: the worst case), timed with CUDA events as eager launches and replayed from a graph."""
    from maya2_native_b200.guards import DeviceGuards, GuardConfig
    dev = torch.device("cuda", 0)
    S = a.seats
    bias = torch.zeros(S + 1, device=dev)
    g = DeviceGuards(GuardConfig(every=1), S, bias)
    for s in range(S):
        g.bind(s, 10 ** 6)
    g.frames[:S] = 99
    g.hist[:S] = torch.randint(0, 2048, (S, g.cfg.hist), device=dev, dtype=torch.int32)
    slots = torch.arange(S, device=dev)
    cb0 = torch.randint(0, 2048, (S,), device=dev)
    code = torch.zeros(S, dtype=torch.long, device=dev)
    reps = 200
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    for _ in range(10):
        g.step(slots, code.zero_(), cb0)
    torch.cuda.synchronize()
    e0.record()
    for _ in range(reps):
        g.step(slots, code, cb0)
    e1.record()
    torch.cuda.synchronize()
    eager = e0.elapsed_time(e1) / reps * 1e3
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        g.step(slots, code, cb0, side)
    torch.cuda.current_stream().wait_stream(side)
    gr = torch.cuda.CUDAGraph()
    with torch.cuda.graph(gr):
        for _ in range(20):
            g.step(slots, code, cb0, torch.cuda.current_stream())
    gr.replay()
    torch.cuda.synchronize()
    e0.record()
    for _ in range(10):
        gr.replay()
    e1.record()
    torch.cuda.synchronize()
    graphed = e0.elapsed_time(e1) / 200 * 1e3
    print(f"guard over {S} seats (every update due): {eager:.2f} us per eager launch, {graphed:.2f} us per graph node")


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("case", choices=("attention", "tick", "gemm", "mimi", "gaps", "overlap", "guard"))
    ap.add_argument("--seats", type=int, default=64)
    ap.add_argument("--layers", type=int, default=2)
    ap.add_argument("--steps", type=int, default=3)
    ap.add_argument("--shape", default="", help="gemm: only this layer of the table (e.g. 'depth.qkv n8')")
    ap.add_argument("--cold", action="store_true", help="gemm: stream the weights from HBM on every launch")
    ap.add_argument("--with", dest="with_", default="mimi",
                    choices=("mimi", "depth", "depth+mimi", "prefill+depth", "depth-halves"),
                    help="overlap: the stage run beside the backbone step (depth+mimi: the Mimi decode beside the "
                         "depth loop; prefill+depth: a backbone prefill of --prompt positions in one free slot "
                         "beside the depth loop; depth-halves: the depth loops of two seat halves, each on its own "
                         "FastDepth handle, beside each other)")
    ap.add_argument("--prompt", type=int, default=350, help="overlap prefill+depth: prompt positions prefilled")
    a = ap.parse_args()
    {"attention": attention, "tick": tick, "gemm": gemm, "mimi": mimi, "gaps": gaps, "overlap": overlap,
     "guard": guard}[a.case](a)


if __name__ == "__main__":
    main()
