"""The decode-only backbone step (m3_backbone_step_decode: each layer's q/k head RMSNorm, RoPE and K/V cache write
run inside its attention launch, serve/fast_backbone.py:62-92 folded into :32-58) against the plain step on the same
state: the same hidden states and the same K/V caches, bit for bit.

Covered: GQA groups 1, 2 and 4; padding rows; few rows whose keys span several splits (only the split that ends at
the row's position writes its K/V); a full batch in one split per row, with the row's own position in the first
copies of a warp and in later ones; decode steps after inline prefills; graphs and eager launches.  The measurement
hook's re-run of a decode step's attention leaves the caches as they are."""
import dataclasses

import numpy as np
import pytest
import torch

from maya2_native_b200 import _lib as L
from maya2_native_b200 import weights as WG
from maya2_native_b200.backbone import StaticBackbone
from maya2_native_b200.config import TINY

pytestmark = pytest.mark.gpu


def pair(g, slots, capacity, buckets, use_graphs):
    W = WG.backbone_weights(g, seed=11)
    out = []
    for decode_form in (True, False):
        sb = StaticBackbone(W, slots, capacity=capacity, ctx_buckets=(256, 512, capacity), batch_buckets=buckets,
                            use_graphs=use_graphs, geom=g)
        sb.decode_form = decode_form
        out.append(sb)
    return out


def fill(pairs, lengths, seed):
    """The same random K/V prefix of lengths[slot] positions in every backbone of the pair."""
    g, dev = pairs[0].geom, pairs[0].device
    gen = torch.Generator(device=dev).manual_seed(seed)
    for slot, n in enumerate(int(n) for n in lengths):
        if n == 0:
            continue
        shape = (1, g.kv_heads, n, g.head_dim)
        kv = [(torch.randn(shape, generator=gen, device=dev).to(torch.bfloat16),
               torch.randn(shape, generator=gen, device=dev).to(torch.bfloat16)) for _ in range(g.layers)]
        for sb in pairs:
            sb.load_prefix(slot, kv, n)


def same_state(a, b):
    """Every real slot's K/V and length (the padding slot's position 0 holds whichever padding row wrote last)."""
    torch.cuda.synchronize()
    n = a.max_slots
    for i in range(a.geom.layers):
        assert torch.equal(a.k[i][:n], b.k[i][:n]), f"K cache of layer {i}"
        assert torch.equal(a.v[i][:n], b.v[i][:n]), f"V cache of layer {i}"
    assert torch.equal(a.lengths, b.lengths) and a.lengths_cpu == b.lengths_cpu


def decode_steps(a, b, slots, n, seed, cuda):
    gen = torch.Generator().manual_seed(seed)
    for _ in range(n):
        x = (torch.randn(len(slots), a.hidden, generator=gen) * 2).to(cuda, torch.bfloat16)
        ya, yb = a.step(slots, x), b.step(slots, x)
        assert torch.equal(ya, yb), float((ya.float() - yb.float()).abs().max())
    same_state(a, b)


def geom(heads, kv_heads):
    return dataclasses.replace(TINY.backbone, heads=heads, kv_heads=kv_heads)


@pytest.mark.parametrize("heads,kv_heads", [(4, 4), (4, 2), (8, 2)])
@pytest.mark.parametrize("use_graphs", [False, True])
def test_few_rows_over_split_keys(cuda, heads, kv_heads, use_graphs):
    """5 rows in an 8-row bucket (3 padding rows) at context 1024: 64-key splits, positions anywhere in them."""
    a, b = pair(geom(heads, kv_heads), 8, 1024, (1, 4, 8), use_graphs)
    lengths = [0, 5, 63, 64, 130, 700, 1000]
    fill((a, b), lengths, seed=heads)
    decode_steps(a, b, [1, 2, 3, 4, 5], 3, seed=1, cuda=cuda)
    decode_steps(a, b, [6, 0, 2], 2, seed=2, cuda=cuda)           # a slot from length 0, and one near capacity
    assert a.device_status() == 0 and b.device_status() == 0
    a.close()
    b.close()


def test_full_batch_one_split_per_row(cuda):
    """100 rows in a 128-row bucket with 8 KV heads: one split per row, each row's own position in a warp's first
    copies (short rows) or in a later one (rows past 128 keys); then a mixed step with inline prompts (plain form
    on both) and decode steps after it."""
    g = geom(16, 8)
    a, b = pair(g, 130, 1024, (8, 128), True)
    rng = np.random.default_rng(3)
    lengths = list(rng.integers(0, 1000, 130))
    fill((a, b), lengths, seed=3)
    slots = [int(s) for s in rng.permutation(130)[:100]]
    decode_steps(a, b, slots, 2, seed=4, cuda=cuda)
    gen = torch.Generator().manual_seed(5)
    free = [s for s in range(130) if s not in slots][:2]
    for s in free:
        a.free(s)
        b.free(s)
    prompts = [(s, (torch.randn(n, g.hidden, generator=gen)).to(cuda, torch.bfloat16)) for s, n in zip(free, (9, 17))]
    x = torch.randn(40, g.hidden, generator=gen).to(cuda, torch.bfloat16)
    da, la = a.step_mixed(slots[:40], x, prompts)
    db, lb = b.step_mixed(slots[:40], x, prompts)
    assert torch.equal(da, db) and all(torch.equal(p, q) for p, q in zip(la, lb))
    decode_steps(a, b, slots[:60] + free, 2, seed=6, cuda=cuda)
    assert a.device_status() == 0 and b.device_status() == 0
    a.close()
    b.close()


def test_measurement_hook_after_a_decode_step_keeps_the_caches(cuda):
    g = geom(4, 2)
    a, b = pair(g, 8, 1024, (8,), False)
    fill((a, b), [3, 70, 500, 900], seed=7)
    decode_steps(a, b, [0, 1, 2, 3], 1, seed=8, cuda=cuda)
    before = [t.clone() for t in a.k + a.v]
    lib = L.load()
    for layer in range(g.layers):
        L.check(lib.m3_backbone_attention(a._handle, layer, 8, 1024, L.stream_ptr()), "m3_backbone_attention")
    torch.cuda.synchronize()
    assert all(torch.equal(x, y) for x, y in zip(before, a.k + a.v))
    assert a.device_status() == 0
    a.close()
    b.close()
