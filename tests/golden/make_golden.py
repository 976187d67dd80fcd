"""Generate the golden fixtures in this directory by running the REFERENCE implementation itself.

Run in a container that has the reference checkout (it is read-only and is never needed at test time):

    python tests/golden/make_golden.py --ref /path/to/maya2-native

The reference's Triton kernels run under the Triton interpreter (TRITON_INTERPRET=1) on CPU tensors, so the fixtures
pin the exact serving path: the fused bf16 backbone (serve/fast_backbone.py, fuse_rope=True), the fused depth body and
its Philox top-k sampler (serve/fast_depth.py, serve/fast_depth_kernels.py), the cb0 sampler with controlled stop
(maya3/engine.py:652-694) and the static-state Mimi decoder (serve/fast_codec.py).  Weights come from
maya2_native_b200.weights (seeded by name), so only inputs and outputs are stored; the tests regenerate the weights.
The reference's hard-coded depth geometry (tts/model/depth_v2.py:45-48, serve/fast_depth.py:26-29) is patched to the
small test geometry before its modules are built.
"""
import argparse
import os
import sys
import types

os.environ["TRITON_INTERPRET"] = "1"
HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, REPO)

import numpy as np  # noqa: E402
import torch  # noqa: E402

from maya2_native_b200 import weights as WG  # noqa: E402
from maya2_native_b200.config import TINY, BackboneGeom, DepthGeom  # noqa: E402

DT = {"fp32": torch.float32, "bf16": torch.bfloat16}


def patch_interpreter_rounding():
    """Triton's GPU backend lowers fp32 -> bf16 casts with round-to-nearest-even (the documented default of
    ``fp_downcast_rounding``); its CPU interpreter truncates instead.  Give the interpreter the device's rounding so
    the fixtures reproduce what the reference's kernels compute on a GPU."""
    import triton.language as tl
    from triton.runtime import interpreter as I
    orig = I.InterpreterBuilder.cast_impl

    def cast_impl(self, src, dst_type):
        if src.dtype.scalar == tl.float32 and dst_type.scalar == tl.bfloat16:
            u = np.ascontiguousarray(src.data, dtype=np.float32).view(np.uint32)
            r = ((u + np.uint32(0x7FFF) + ((u >> 16) & np.uint32(1))) >> 16).astype(np.uint16)
            return I.TensorHandle(r, dst_type.scalar)
        return orig(self, src, dst_type)
    I.InterpreterBuilder.cast_impl = cast_impl


def np32(t):
    return t.detach().float().cpu().numpy()


def load_named(module, prefix, seed=0):
    """Fill every parameter/buffer of a reference module from the seeded generator under prefix+name."""
    sd = module.state_dict()
    new = {k: WG.make(prefix + k, v.shape, seed).to(v.dtype) for k, v in sd.items() if k != "lm_head.weight"}
    module.load_state_dict(new, strict=False)   # lm_head is tied to the embedding


# ------------------------------------------------------------------------------------------------ backbone
def qwen3(g: BackboneGeom, dtype):
    from transformers import Qwen3Config, Qwen3ForCausalLM
    cfg = Qwen3Config(hidden_size=g.hidden, num_hidden_layers=g.layers, num_attention_heads=g.heads,
                      num_key_value_heads=g.kv_heads, head_dim=g.head_dim, intermediate_size=g.ffn,
                      vocab_size=g.vocab, rms_norm_eps=g.eps, tie_word_embeddings=True,
                      rope_parameters={"rope_theta": g.rope_theta, "rope_type": "default"})
    lm = Qwen3ForCausalLM(cfg)
    load_named(lm, "")
    return lm.to(dtype).eval()


def gen_backbone(dtype):
    from serve.fast_backbone import StaticBackbone
    g = TINY.backbone
    lm = qwen3(g, DT[dtype])
    fused = dtype == "bf16"
    sb = StaticBackbone(types.SimpleNamespace(lm=lm), 3, capacity=64, ctx_buckets=(64,), use_graphs=False,
                        attention="triton" if fused else "gather", fuse_rope=fused)
    rng = torch.Generator().manual_seed(11)
    calls = [  # (slots, offsets): inline prefill, decode, then mixed decode + prefill
        ([0] * 5 + [1] * 3, list(range(5)) + list(range(3))),
        ([0, 1, 2], [0, 0, 0]), ([0, 1, 2], [0, 0, 0]), ([2, 0, 1], [0, 0, 0]),
        ([0, 1] + [2] * 4, [0, 0, 0, 1, 2, 3]),
        ([1, 2, 0], [0, 0, 0]),
    ]
    out = {}
    with torch.inference_mode():
        for i, (slots, offs) in enumerate(calls):
            x = torch.randn(len(slots), g.hidden, generator=rng).to(DT[dtype])
            s = torch.tensor(slots)
            y = sb._forward(s, x, torch.ones(len(slots), dtype=torch.long), 64, torch.tensor(offs))
            out[f"slots{i}"] = np.array(slots)
            out[f"offsets{i}"] = np.array(offs)
            out[f"x{i}"] = np32(x)
            out[f"out{i}"] = np32(y)
        out["lengths"] = sb.lengths.numpy()
        out["k_last"] = np32(sb.k[-1][:3, :, :12])
        out["v_last"] = np32(sb.v[-1][:3, :, :12])
    np.savez_compressed(os.path.join(HERE, f"backbone_tiny_{dtype}.npz"), **out)


# ------------------------------------------------------------------------------------------------ cb0 sampler
def gen_cb0():
    from maya3.engine import Engine
    g = TINY.backbone
    B, m = 5, 6
    lin = torch.nn.Linear(g.hidden, g.n_cb0, bias=False)
    lin.weight.data.copy_(WG.make("cb0_head.weight", (g.n_cb0, g.hidden)))
    lin = lin.to(torch.bfloat16)
    st = types.SimpleNamespace(
        model=types.SimpleNamespace(backbone=types.SimpleNamespace(cb0_logits=lin)),
        cfg=types.SimpleNamespace(cb0_rep_win=12, cb0_rep=0.8),
        _any_rep=True, _any_top_p=True,
        temp_t=torch.tensor([0.9, 0.5, 1.3, 0.9, 0.7, 0.9]),
        topk_t=torch.tensor([64, 1, 2049, 200, 10, 64]),
        topp_t=torch.tensor([1.0, 1.0, 1.0, 0.8, 1.0, 1.0]),
        rep_t=torch.tensor([0.8, 0.0, 2.0, 0.8, 0.8, 0.8]),
        aeos_bias=torch.tensor([0.0, 0.0, 3.0, 0.0, 12.0, 0.0]),
        seed_t=torch.tensor([17, 99, 12345, 7, 2 ** 31 - 2, 0], dtype=torch.int32),
        ctr_t=torch.tensor([0, 5, 1499, 3, 0, 0], dtype=torch.int32),
        hist_t=torch.full((m, 12), -1, dtype=torch.long),
        frames_t=torch.tensor([0, 10, 40, 3, 8, 0]), min_t=torch.tensor([4, 4, 4, 4, 4, 0]),
        hazard_t=torch.tensor([0.0, 0.1, 0.5, 0.3, 0.0, 0.0]))
    hist_rng = torch.Generator().manual_seed(3)
    st.hist_t[:, 4:] = torch.randint(0, 64, (m, 8), generator=hist_rng)
    out = {k: v.numpy().copy() for k, v in vars(st).items() if torch.is_tensor(v)}
    out = {"init_" + k: v for k, v in out.items()}
    rng = torch.Generator().manual_seed(5)
    idx = torch.tensor([0, 1, 2, 3, 4])
    with torch.inference_mode():
        for it in range(3):
            h = (torch.randn(B, g.hidden, generator=rng) * 1.0).to(torch.bfloat16)
            out[f"h{it}"] = np32(h)
            out[f"logits{it}"] = np32(lin(h).float())
            code, cb0 = Engine._cb0(st, h, idx)
            out[f"code{it}"] = code.numpy()
            out[f"cb0{it}"] = cb0.numpy()
    for k in ("ctr_t", "hist_t", "frames_t", "hazard_t"):
        out["final_" + k] = getattr(st, k).numpy()
    np.savez_compressed(os.path.join(HERE, "cb0_sampler.npz"), **out)


def gen_topk():
    from serve.fast_depth_kernels import topk_sample
    rng = torch.Generator().manual_seed(9)
    out = {}
    lg = torch.randn(6, 2048, generator=rng) * 3
    lg[5, 100:110] = lg[5].max() + 1          # ties at the top
    seeds = torch.tensor([1, 2, 3, 4, 5, 2 ** 30], dtype=torch.int32)
    ctrs = torch.tensor([0, 1, 2, 100, 1499, 7], dtype=torch.int32)
    out["logits"], out["seeds"], out["ctrs"] = lg.numpy(), seeds.numpy(), ctrs.numpy()
    for level in (1, 5, 31):
        for k in (1, 50, 64, 2048):
            out[f"s_l{level}_k{k}"] = topk_sample(lg, seeds, level, 0.7, k, False, ctr_t=ctrs).numpy()
        out[f"g_l{level}"] = topk_sample(lg, seeds, level, 0.8, 50, True, ctr_t=ctrs).numpy()
    lb = lg.to(torch.bfloat16)
    out["logits_bf16"] = np32(lb)
    out["s_bf16"] = topk_sample(lb, seeds, 3, 0.8, 50, False, ctr_t=ctrs).numpy()
    np.savez_compressed(os.path.join(HERE, "topk_sampler.npz"), **out)


# ------------------------------------------------------------------------------------------------ depth
def patch_depth(g: DepthGeom):
    import serve.fast_depth as FD
    import tts.model.depth_v2 as DV
    gol = list(g.group_of_level)
    for mod in (DV, FD):
        mod.D, mod.H, mod.LAYERS, mod.GROUP_OF_LEVEL = g.d, g.heads, g.layers, gol
    DV.FFN, DV.RANK, DV.N_GROUPS = g.ffn, g.rank, g.n_groups
    FD.HEAD, FD.N_LEVELS = g.d // g.heads, g.n_q


def depth_model(g: DepthGeom, dtype):
    from tts.model.audio_io import AudioInputEmbed
    from tts.model.depth_v2 import DepthV2
    patch_depth(g)
    depth = DepthV2(d_backbone=g.d_backbone, n_q=g.n_q, n_codes=g.n_codes)
    load_named(depth, "depth.")
    audio_in = AudioInputEmbed(g.d_backbone, n_q=g.n_q, n_codes=g.n_codes)
    load_named(audio_in, "audio_in.")
    return types.SimpleNamespace(depth=depth.eval(), audio_in=audio_in.to(DT[dtype]).eval())


def gen_depth(name, g: DepthGeom, dtype, frames=2):
    from serve.fast_depth import FastDepth
    model = depth_model(g, dtype)
    B = 3
    out = {}
    rng = torch.Generator().manual_seed(21)
    for greedy in (True, False):
        fd = FastDepth(model, B, dtype=DT[dtype], temp=0.8, top_k=50, batch_buckets=(B,), seed=7, greedy=greedy,
                       fused=True)
        mems = torch.randn(B, 1, 1, g.d, generator=torch.Generator().manual_seed(4))
        for s in range(B):
            fd.set_speaker(s, mems[s], torch.ones(1, 1, dtype=torch.bool))
        fd.row_seed[:B] = torch.tensor([11, 22, 2 ** 31 - 3], dtype=torch.int32)
        out["mems"] = mems.numpy()
        tag = "g" if greedy else "s"
        slots = torch.tensor([2, 0, 1])
        with torch.inference_mode():
            for f in range(frames):
                h = torch.randn(B, g.d_backbone, generator=rng).to(DT[dtype])
                cb0 = torch.randint(0, g.n_codes, (B,), generator=rng)
                codes, fb = fd._fn(slots, h, cb0)
                out[f"{tag}_h{f}"], out[f"{tag}_cb0_{f}"] = np32(h), cb0.numpy()
                out[f"{tag}_codes{f}"], out[f"{tag}_fb{f}"] = codes.numpy(), np32(fb)
        out[f"{tag}_row_ctr"] = fd.row_ctr.numpy()
        out["slots"] = slots.numpy()
    np.savez_compressed(os.path.join(HERE, f"{name}_{dtype}.npz"), **out)


# ------------------------------------------------------------------------------------------------ mimi
def mimi_model(g, dtype):
    from transformers import MimiConfig, MimiModel
    cfg = MimiConfig(hidden_size=g.hidden, num_quantizers=g.n_q, num_semantic_quantizers=g.n_semantic,
                     codebook_size=g.codebook_size, codebook_dim=g.codebook_dim,
                     vector_quantization_hidden_dimension=g.codebook_dim, num_hidden_layers=g.layers,
                     num_attention_heads=g.heads, num_key_value_heads=g.heads, intermediate_size=g.ffn,
                     sliding_window=g.window, upsampling_ratios=list(g.ratios), num_filters=g.num_filters,
                     upsample_groups=g.hidden,
                     sampling_rate=int(12.5 * 2 * np.prod(g.ratios)), frame_rate=12.5,
                     rope_parameters={"rope_theta": g.rope_theta, "rope_type": "default"})
    m = MimiModel(cfg)
    load_named(m, "mimi.")
    for mod in m.modules():
        if hasattr(mod, "_embed"):
            mod._embed = None
    return m.to(DT[dtype]).eval()


def gen_mimi(dtype, frames=24):
    from serve.fast_codec import StaticMimi
    g = TINY.mimi
    m = mimi_model(g, dtype)
    sm = StaticMimi(m, 3, ring=g.ring)
    rng = torch.Generator().manual_seed(31)
    out = {}
    with torch.inference_mode():
        for f in range(frames):
            slots = [0, 1] if f < 5 else ([0, 1, 2] if f % 2 else [2, 1, 0])
            if f == 5:
                sm.reset(2)
            if f == 14:
                sm.reset(1)
            codes = torch.randint(0, g.codebook_size, (len(slots), g.n_q), generator=rng)
            pcm = sm._forward(torch.tensor(slots), codes[:, :, None])
            out[f"slots{f}"], out[f"codes{f}"], out[f"pcm{f}"] = np.array(slots), codes.numpy(), np32(pcm[:, 0])
    np.savez_compressed(os.path.join(HERE, f"mimi_tiny_{dtype}.npz"), **out)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--ref", required=True, help="path of a reference checkout (read-only; used only here)")
    ap.add_argument("--only", default="")
    a = ap.parse_args()
    sys.path.insert(0, a.ref)
    patch_interpreter_rounding()
    torch.manual_seed(0)
    jobs = {
        "backbone": lambda: [gen_backbone(d) for d in ("fp32", "bf16")],
        "cb0": gen_cb0, "topk": gen_topk,
        "depth": lambda: [gen_depth("depth_tiny", TINY.depth, d) for d in ("fp32", "bf16")],
        "depth_grouped": lambda: gen_depth(
            "depth_grouped", DepthGeom(layers=2, d=128, heads=2, ffn=256, n_q=12, rank=16, d_backbone=256), "fp32"),
        "mimi": lambda: [gen_mimi(d) for d in ("fp32", "bf16")],
    }
    for name, fn in jobs.items():
        if a.only and name not in a.only.split(","):
            continue
        print("generating", name, flush=True)
        fn()


if __name__ == "__main__":
    main()
