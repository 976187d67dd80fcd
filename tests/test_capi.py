"""The C ABI library loads and exports every entry point include/maya3_b200.h declares (no GPU calls), and the
host-side layout logic agrees with the reference's.  CPU only."""
import os
import re

import pytest

from conftest import REPO
from maya2_native_b200 import _lib as L
from maya2_native_b200.config import BASELINE, TINY
from maya2_native_b200.weights import mimi_decoder_layout

HEADER = os.path.join(REPO, "include", "maya3_b200.h")


def declared():
    text = open(HEADER).read()
    return sorted(set(re.findall(r"^M3_API [^(]*?\b(m3_\w+)\(", text, flags=re.M)))


@pytest.fixture(scope="module")
def lib():
    if not os.path.exists(L.LIB_PATH):
        from maya2_native_b200.build import build
        build()
    return L.load()


def test_every_declared_symbol_is_exported(lib):
    names = declared()
    assert len(names) >= 20
    missing = [n for n in names if not hasattr(lib, n)]
    assert not missing, missing


def test_binding_covers_the_header():
    assert sorted(L.SIGNATURES) == declared()


def test_version_and_error_string(lib):
    assert lib.m3_version() >= 1
    assert isinstance(lib.m3_last_error(), bytes)


def _mimi_cfg(g, max_slots=4):
    return L.MimiConfig(g.hidden, g.n_q, g.n_semantic, g.codebook_size, g.codebook_dim, g.layers, g.heads, g.ffn,
                        g.window, g.ring, len(g.ratios), (L.i32 * 8)(*(list(g.ratios) + [0] * (8 - len(g.ratios)))),
                        g.num_filters, g.kernel, g.last_kernel, g.res_kernel, g.compress, g.upsample_stride,
                        max_slots, max_slots, g.norm_eps)


def test_mimi_state_row_matches_reference_layout(lib):
    """StaticMimi keeps 12,672 state elements per slot at this geometry (serve/fast_codec.py:52-63, _plan :81-96):
    the same histories and tails, here channels-last."""
    assert lib.m3_mimi_state_elems(_mimi_cfg(BASELINE.mimi)) == 12672
    g = TINY.mimi
    ref = g.upsample_stride * g.hidden + (g.kernel - 1) * g.hidden
    for _, kind, cin, cout, k, stride in mimi_decoder_layout(g):
        if kind == "convt":
            ref += stride * cout
        elif kind == "resnet":
            ref += (k - 1) * cin
        elif kind == "conv" and cin == g.num_filters:
            ref += (k - 1) * cin
    assert lib.m3_mimi_state_elems(_mimi_cfg(g)) == ref


def test_geometry_constants():
    g = BASELINE.backbone
    assert g.kv_bytes_per_token() == 112 * 1024          # docs/ENGINE.md:167
    assert BASELINE.mimi.samples_per_frame == 1920
    assert BASELINE.depth.group_of_level == (None, 0, 1, 2, 3, 4, 5, 6)
    assert BASELINE.depth.head_dim == 128


# ---- argument validation at the boundary: these calls return their status before touching the device, so they
# run on CPU; the binding raises what the reference raises (ValueError for shapes/arguments, IndexError for slots).
def test_bad_arguments_map_to_reference_exceptions(lib):
    with pytest.raises(ValueError, match="bad shape"):
        L.check(lib.m3_gemm_bf16(None, 8, None, 8, None, 8, 4, 0, 8, 0, None), "m3_gemm_bf16")
    with pytest.raises(ValueError, match="null argument"):
        L.check(lib.m3_topk_sample(None, 1, 4, 2048, None, None, 1, 1.0, 50, 0, None, None), "m3_topk_sample")
    with pytest.raises(ValueError, match="null argument"):
        L.check(lib.m3_tick_create(None, L.vp()), "m3_tick_create")
    with pytest.raises(ValueError):
        L.check(lib.m3_backbone_step(None, None, None, None, None, None, 1, 1, None), "m3_backbone_step")
    with pytest.raises(ValueError, match="null handle"):
        L.check(lib.m3_mimi_set_sm_budget(None, 37), "m3_mimi_set_sm_budget")
    with pytest.raises(ValueError, match="null argument"):
        L.check(lib.m3_slot_reset(None, None, None), "m3_slot_reset")
    with pytest.raises(ValueError, match="activation"):
        L.check(lib.m3_gemm_bf16_act(None, 8, None, 8, None, 8, 1, 8, 8, 3, None), "m3_gemm_bf16_act")


def test_unsupported_geometries_are_rejected(lib):
    g = BASELINE.backbone
    cfg = L.BackboneConfig(g.layers, g.hidden, g.heads, g.kv_heads, 64, g.ffn, 4, 512, 16, g.eps)  # head_dim 64
    w = L.BackboneWeights()
    h = L.vp()
    rc = lib.m3_backbone_create(cfg, w, h)
    assert rc == L.M3_ERR_UNSUPPORTED and b"head_dim" in lib.m3_last_error()
    bad = _mimi_cfg(BASELINE.mimi)
    bad.n_ratios = 0
    assert lib.m3_mimi_state_elems(bad) == -1
    assert lib.m3_mimi_create(bad, L.MimiWeights(), L.vp()) == L.M3_ERR_ARG


def test_status_codes_of_the_binding():
    assert L.DEV_STATUS[4] == "kernel wait timed out"
    with pytest.raises(IndexError):
        L.check(L.M3_ERR_RANGE, "x")
    with pytest.raises(L.M3Error):
        L.check(L.M3_ERR_CUDA, "x")


def test_guard_and_prefix_entry_points_validate_before_the_device(lib):
    """m3_guard_step / m3_tick_set_guard refuse configurations outside their limits (stall or period window longer
    than the history, pmax >= period_win, a history above 128, a bad mode, null state arrays) and the prefix copies
    refuse a null handle -- all before any device work."""
    fake = L.GuardState(*([8] * 8))                      # non-null pointers that are never dereferenced
    ok = dict(loop=1, stall=32, period_win=64, period_thr=0.7, pmin=2, pmax=16, start=32, every=2, mode=0, boost=4.0,
              backstop=24, hist=96, max_windows=4, max_slots=8)
    for bad in (dict(hist=200), dict(stall=100), dict(period_win=100), dict(pmax=64), dict(mode=2), dict(every=0),
                dict(pmin=0), dict(max_slots=0)):
        cfg = L.GuardConfig(**{**ok, **bad})
        assert lib.m3_guard_step(cfg, fake, None, None, None, 0, None) == L.M3_ERR_ARG, bad
    cfg = L.GuardConfig(**ok)
    assert lib.m3_guard_step(cfg, L.GuardState(), None, None, None, 0, None) == L.M3_ERR_ARG   # null state
    assert lib.m3_guard_step(cfg, fake, None, None, None, 4, None) == L.M3_ERR_ARG             # null slots
    assert lib.m3_guard_step(cfg, fake, 8, 8, 8, 0, None) == L.M3_OK                           # nothing to do
    assert lib.m3_tick_set_guard(None, cfg, fake) == L.M3_ERR_ARG
    assert lib.m3_backbone_load_prefix(None, 0, 16, 4, None) == L.M3_ERR_ARG
    assert lib.m3_backbone_save_prefix(None, 0, 16, 4, None) == L.M3_ERR_ARG
