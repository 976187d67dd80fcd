"""ctypes binding of libm3b200.so (include/maya3_b200.h).

There is no fallback: importing the product path on a machine without the built library raises immediately.
"""
from __future__ import annotations

import ctypes as C
import os
import threading

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libm3b200.so")

M3_OK, M3_ERR_ARG, M3_ERR_CUDA, M3_ERR_RANGE, M3_ERR_UNSUPPORTED = 0, -1, -2, -3, -4
DEV_STATUS = {0: "ok", 1: "slot out of range", 2: "position reached capacity", 3: "code out of range",
              4: "kernel wait timed out"}

vp = C.c_void_p
i32 = C.c_int32
i64 = C.c_int64
f32 = C.c_float
P = C.POINTER


class BackboneConfig(C.Structure):
    _fields_ = [("layers", i32), ("hidden", i32), ("heads", i32), ("kv_heads", i32), ("head_dim", i32),
                ("ffn", i32), ("max_slots", i32), ("capacity", i32), ("max_rows", i32), ("eps", f32)]


class BackboneWeights(C.Structure):
    _fields_ = [("in_norm", P(vp)), ("wqkv", P(vp)), ("q_norm", P(vp)), ("k_norm", P(vp)), ("wo", P(vp)),
                ("post_norm", P(vp)), ("wgu", P(vp)), ("wdown", P(vp)), ("final_norm", vp), ("cos", vp),
                ("sin", vp), ("k_cache", P(vp)), ("v_cache", P(vp)), ("lengths", vp)]


class Cb0Config(C.Structure):
    _fields_ = [("hidden", i32), ("n_cls", i32), ("max_slots", i32), ("max_rows", i32), ("rep_win", i32)]


class Cb0State(C.Structure):
    _fields_ = [("head", vp), ("frames", vp), ("min_frames", vp), ("hazard", vp), ("aeos_bias", vp), ("temp", vp),
                ("top_k", vp), ("top_p", vp), ("rep", vp), ("seed", vp), ("ctr", vp), ("hist", vp)]


class SlotState(C.Structure):
    _fields_ = [("frames", vp), ("min_frames", vp), ("hazard", vp), ("aeos_bias", vp), ("seed", vp), ("ctr", vp),
                ("hist", vp), ("hist_len", i32), ("temp", vp), ("top_k", vp), ("top_p", vp), ("rep", vp),
                ("row_seed", vp), ("row_ctr", vp), ("cross_const", vp), ("cross_elems", i32), ("lengths", vp),
                ("max_slots", i32)]


class SlotInit(C.Structure):
    _fields_ = [("slot", i32), ("seed", i32), ("row_seed", i32), ("min_frames", i32), ("top_k", i64),
                ("length", i64), ("temp", f32), ("top_p", f32), ("rep", f32), ("cross_src", vp)]


class GuardConfig(C.Structure):
    _fields_ = [("loop", i32), ("stall", i32), ("period_win", i32), ("period_thr", C.c_double), ("pmin", i32),
                ("pmax", i32), ("start", i32), ("every", i32), ("mode", i32), ("boost", f32), ("backstop", i32),
                ("hist", i32), ("max_windows", i32), ("max_slots", i32)]


class GuardState(C.Structure):
    _fields_ = [("frames", vp), ("cap", vp), ("boost_at", vp), ("n_boost", vp), ("hist", vp), ("n_windows", vp),
                ("windows", vp), ("aeos_bias", vp)]


class DepthConfig(C.Structure):
    _fields_ = [("layers", i32), ("d", i32), ("heads", i32), ("ffn", i32), ("n_q", i32), ("n_codes", i32),
                ("d_backbone", i32), ("n_groups", i32), ("group_of_level", i32 * 64), ("max_slots", i32),
                ("max_rows", i32), ("ln_eps", f32), ("inv_temp", f32), ("top_k", i32), ("greedy", i32)]


class DepthWeights(C.Structure):
    _fields_ = [("in_proj", vp), ("embed", vp), ("level0", vp), ("n1_w", P(vp)), ("n1_b", P(vp)),
                ("n2_w", P(vp)), ("n2_b", P(vp)), ("qkv", P(vp)), ("o", P(vp)), ("f1", P(vp)), ("f2", P(vp)),
                ("norm_w", vp), ("norm_b", vp), ("heads", P(vp)), ("cross_kv", P(vp)), ("cross_o", P(vp)),
                ("audio_table", vp), ("audio_norm", vp), ("cross_const", vp), ("row_seed", vp), ("row_ctr", vp)]


class MimiConfig(C.Structure):
    _fields_ = [("hidden", i32), ("n_q", i32), ("n_semantic", i32), ("codebook_size", i32), ("codebook_dim", i32),
                ("layers", i32), ("heads", i32), ("ffn", i32), ("window", i32), ("ring", i32), ("n_ratios", i32),
                ("ratios", i32 * 8), ("num_filters", i32), ("kernel", i32), ("last_kernel", i32),
                ("res_kernel", i32), ("compress", i32), ("upsample_stride", i32), ("max_slots", i32),
                ("max_rows", i32), ("norm_eps", f32)]


class MimiWeights(C.Structure):
    _fields_ = [("codebooks", vp), ("proj_sem", vp), ("proj_ac", vp), ("upsample", vp),
                ("ln1_w", P(vp)), ("ln1_b", P(vp)), ("wqkv", P(vp)), ("wo", P(vp)), ("ln2_w", P(vp)),
                ("ln2_b", P(vp)), ("fc1", P(vp)), ("fc2", P(vp)), ("ls1", P(vp)), ("ls2", P(vp)),
                ("inv_freq", vp), ("conv0_w", vp), ("conv0_b", vp), ("convt_w", P(vp)), ("convt_b", P(vp)),
                ("res1_w", P(vp)), ("res1_b", P(vp)), ("res2_w", P(vp)), ("res2_b", P(vp)), ("final_w", vp),
                ("final_b", vp), ("conv_state", vp), ("kv", vp), ("key_pos", vp), ("tokens", vp)]


class TickConfig(C.Structure):
    _fields_ = [("bb", vp), ("cb0", vp), ("depth", vp), ("mimi", vp), ("embed", vp), ("vocab", i64),
                ("feedback", vp), ("hidden", i32), ("max_rows", i32), ("max_seats", i32), ("n_q", i32), ("spf", i32),
                ("max_slots", i32)]


# name -> (restype, argtypes); every entry point declared in include/maya3_b200.h
SIGNATURES = {
    "m3_last_error": (C.c_char_p, []),
    "m3_version": (C.c_int, []),
    "m3_launch_count": (i64, []),
    "m3_gemm_bf16": (C.c_int, [vp, i64, vp, i64, vp, i64, i32, i32, i32, i32, vp]),
    "m3_gemm_bf16_act": (C.c_int, [vp, i64, vp, i64, vp, i64, i32, i32, i32, i32, vp]),
    "m3_backbone_create": (C.c_int, [P(BackboneConfig), P(BackboneWeights), P(vp)]),
    "m3_backbone_destroy": (C.c_int, [vp]),
    "m3_backbone_step": (C.c_int, [vp, vp, vp, vp, vp, vp, i32, i32, vp]),
    "m3_backbone_status": (C.c_int, [vp, P(i32), i32]),
    "m3_backbone_attention": (C.c_int, [vp, i32, i32, i32, vp]),
    "m3_backbone_attention_selftest": (C.c_int, [vp, i32, i32, i32, vp]),
    "m3_cb0_create": (C.c_int, [P(Cb0Config), P(Cb0State), P(vp)]),
    "m3_cb0_destroy": (C.c_int, [vp]),
    "m3_cb0_step": (C.c_int, [vp, vp, vp, vp, vp, i32, i32, i32, vp]),
    "m3_cb0_sample_logits": (C.c_int, [vp, vp, vp, vp, vp, i32, i32, i32, vp]),
    "m3_cb0_step_noalloc": (C.c_int, [P(Cb0Config), P(Cb0State), vp, vp, vp, vp, i32, i32, i32, vp]),
    "m3_cb0_noalloc_status": (C.c_int, [P(i32), i32]),
    "m3_cb0_status": (C.c_int, [vp, P(i32), i32]),
    "m3_cb0_copy_logits": (C.c_int, [vp, vp, i32, vp]),
    "m3_depth_debug_logits": (C.c_int, [vp, vp, i64]),
    "m3_depth_create": (C.c_int, [P(DepthConfig), P(DepthWeights), P(vp)]),
    "m3_depth_destroy": (C.c_int, [vp]),
    "m3_depth_set_speaker": (C.c_int, [vp, i32, vp, f32, vp]),
    "m3_depth_step": (C.c_int, [vp, vp, vp, vp, vp, vp, i32, vp]),
    "m3_topk_sample": (C.c_int, [vp, i32, i32, i32, vp, vp, i32, f32, i32, i32, vp, vp]),
    "m3_depth_status": (C.c_int, [vp, P(i32), i32]),
    "m3_mimi_state_elems": (i64, [P(MimiConfig)]),
    "m3_mimi_create": (C.c_int, [P(MimiConfig), P(MimiWeights), P(vp)]),
    "m3_mimi_destroy": (C.c_int, [vp]),
    "m3_mimi_reset": (C.c_int, [vp, i32, i32, vp]),
    "m3_mimi_decode": (C.c_int, [vp, vp, vp, vp, i32, vp]),
    "m3_mimi_status": (C.c_int, [vp, P(i32), i32]),
    "m3_mimi_set_sm_budget": (C.c_int, [vp, i32]),
    "m3_mimi_convt": (C.c_int, [vp, i32, i32, P(C.c_int64), vp]),
    "m3_selftest_timeout": (C.c_int, [i32, P(i32)]),
    "m3_gelu_bf16": (C.c_int, [vp, i64, vp]),
    "m3_pack_readout": (C.c_int, [vp, vp, vp, vp, i32, i32, vp]),
    "m3_tick_create": (C.c_int, [P(TickConfig), P(vp)]),
    "m3_tick_destroy": (C.c_int, [vp]),
    "m3_tick_run": (C.c_int, [vp, vp, i32, i32, i32, i32, i32, vp, vp]),
    "m3_slot_reset": (C.c_int, [P(SlotState), P(SlotInit), vp]),
    "m3_tick_run_main": (C.c_int, [vp, vp, i32, i32, i32, i32, i32, vp]),
    "m3_tick_stage_codec": (C.c_int, [vp, vp, i32, i32, i32, vp]),
    "m3_tick_run_codec": (C.c_int, [vp, i32, i32, vp, vp]),
    "m3_tick_outputs": (C.c_int, [vp, P(vp), P(vp), P(vp)]),
    "m3_tick_status": (C.c_int, [vp, P(i32), i32]),
    "m3_backbone_save_prefix": (C.c_int, [vp, i32, vp, i32, vp]),
    "m3_backbone_load_prefix": (C.c_int, [vp, i32, vp, i32, vp]),
    "m3_guard_step": (C.c_int, [P(GuardConfig), P(GuardState), vp, vp, vp, i32, vp]),
    "m3_tick_set_guard": (C.c_int, [vp, P(GuardConfig), P(GuardState)]),
}

_lock = threading.Lock()
_lib = None


def load(path: str = LIB_PATH):
    """Load and declare the library once; raises if it is missing (the product path has no CPU fallback)."""
    global _lib
    with _lock:
        if _lib is None:
            if not os.path.exists(path):
                raise RuntimeError(f"{path} is not built; run `python -m maya2_native_b200.build` "
                                   "(the CUDA extension is required: there is no fallback path)")
            lib = C.CDLL(path)
            for name, (res, args) in SIGNATURES.items():
                if hasattr(lib, name):
                    fn = getattr(lib, name)
                    fn.restype, fn.argtypes = res, args
            _lib = lib
        return _lib


class M3Error(RuntimeError):
    pass


def check(rc: int, what: str = ""):
    if rc == M3_OK:
        return
    msg = (load().m3_last_error() or b"").decode(errors="replace")
    text = f"{what}: {msg}" if what else msg
    if rc == M3_ERR_ARG:
        raise ValueError(text)
    if rc == M3_ERR_RANGE:
        raise IndexError(text)
    raise M3Error(f"[{rc}] {text}")


def ptr_array(ptrs):
    arr = (vp * len(ptrs))(*[int(p) for p in ptrs])
    return arr


def stream_ptr(stream=None) -> int:
    import torch
    s = stream if stream is not None else torch.cuda.current_stream()
    return int(s.cuda_stream)


def dptr(t) -> int:
    return 0 if t is None else int(t.data_ptr())
