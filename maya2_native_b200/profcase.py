"""Small GPU cases for Nsight Compute captures: a few GB on the device, inputs still far larger than L2.

    python -m maya2_native_b200.profcase attention [--seats 64] [--layers 2] [--steps 3]
    python -m maya2_native_b200.profcase tick [--seats 64] [--steps 3]

attention: the backbone step over `seats` decode rows at the configs[2] KV-length distribution (mean ~790 keys),
           benchmark width, `layers` layers (2 layers x 64 seats ~ 1 GB of K/V); run under
           `ncu -k regex:attn_split -c 3`.
tick:      the full engine tick at the benchmark geometry with fewer seats.
"""
from __future__ import annotations

import argparse
import dataclasses

import numpy as np
import torch


def _lengths(n, rng):
    P = rng.integers(64, 513, n)
    T = np.sqrt(rng.uniform(100 ** 2, 1500 ** 2, n)).astype(np.int64)
    return P + (rng.random(n) * T).astype(np.int64)


@torch.inference_mode()
def attention(a):
    from . import weights as WG
    from .backbone import StaticBackbone
    from .config import BASELINE
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
    for _ in range(a.steps):
        sb.step(list(range(a.seats)), x)
    torch.cuda.synchronize()
    print(f"attention case: {a.seats} seats, {a.layers} layers, mean keys {L.mean():.0f}")


@torch.inference_mode()
def tick(a):
    from . import weights as WG
    from .config import BASELINE
    from .engine import TickConfig, TickEngine
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


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("case", choices=("attention", "tick"))
    ap.add_argument("--seats", type=int, default=64)
    ap.add_argument("--layers", type=int, default=2)
    ap.add_argument("--steps", type=int, default=3)
    a = ap.parse_args()
    {"attention": attention, "tick": tick}[a.case](a)


if __name__ == "__main__":
    main()
