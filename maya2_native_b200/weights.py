"""Seeded random-init weights under the reference's own state-dict names.

There is no checkpoint on either machine, so both sides of every parity check (this package's CUDA path, the CPU
oracle, and -- in the fixture generator only -- the reference's PyTorch modules) consume the same tensors, produced
here from (global seed, tensor name, shape) alone.  Each tensor has its own generator seeded from a CRC of its name,
so a tensor's values do not depend on which other tensors were generated or in what order.

Names follow the reference's modules: the HF ``Qwen3ForCausalLM`` state dict plus ``cb0_head.weight`` for the backbone
(tts/model/backbone.py:83), ``DepthV2`` (tts/model/depth_v2.py:216-237) and ``AudioInputEmbed``
(tts/model/audio_io.py:17-25) under ``depth.`` / ``audio_in.``, and the decoder half of HF ``MimiModel`` under
``mimi.``.

Distributions: norm weights 1 + 0.1 N(0,1), norm/conv biases 0.05 N(0,1), embedding-like tables 0.02 N(0,1) (the
reference's own init), Mimi codebooks N(0,1) with cluster_usage = 1, layer scales 0.2 (1 + 0.1 N), every other
matrix N(0,1)/sqrt(fan_in) so activations keep unit scale through the stacks.
"""
from __future__ import annotations

import zlib

import torch

from .config import BackboneGeom, DepthGeom, MimiGeom

_TABLES = ("embed_tokens.weight", "code_lo.weight", "level_emb.weight", "audio_in.table.weight", "aeos_in",
           "null_mem")


def _kind(name: str, shape: tuple) -> str:
    if name.endswith(("cluster_usage", "initialized")):
        return "ones"
    if name.endswith("codebook.embed_sum"):
        return "randn"
    if name.endswith(_TABLES):
        return "table"
    if name.endswith("layer_scale.scale"):
        return "scale"
    leaf = name.rsplit(".", 2)
    owner = leaf[-2] if len(leaf) >= 2 else ""
    is_norm = "norm" in owner or owner in ("n", "n1", "n2")
    if is_norm and name.endswith(".weight"):
        return "norm_w"
    if name.endswith(".bias"):
        return "bias"
    return "matrix"


def _fan_in(shape: tuple) -> int:
    if len(shape) == 3:
        cin, second, k = shape
        if k % 2 == 0:                     # ConvTranspose1d [C_in, C_out/groups, 2*stride]: two taps reach each output
            return 2 if second == 1 else 2 * cin
        return second * k                  # Conv1d [C_out, C_in, k]
    if len(shape) == 2:
        return shape[1]
    return 1


def make(name: str, shape, seed: int = 0, device=None) -> torch.Tensor:
    """The fp32 tensor for ``name`` at ``shape``: deterministic on CPU (the default, shared with the oracle) for a
    fixed torch build; ``device='cuda'`` draws the same distribution from the device generator (fast, for timing
    runs that need no oracle)."""
    shape = tuple(int(s) for s in shape)
    kind = _kind(name, shape)
    dev = torch.device(device) if device is not None else torch.device("cpu")
    if kind == "ones":
        return torch.ones(shape, device=dev)
    g = torch.Generator(device=dev).manual_seed((int(seed) * 1000003 + zlib.crc32(name.encode())) % (1 << 62))
    r = torch.randn(shape, generator=g, device=dev)
    if kind == "randn":
        return r
    if kind == "table":
        return r * 0.02
    if kind == "scale":
        return 0.2 * (1 + 0.1 * r)
    if kind == "norm_w":
        return 1 + 0.1 * r
    if kind == "bias":
        return 0.05 * r
    return r / (_fan_in(shape) ** 0.5)


def backbone_shapes(g: BackboneGeom) -> dict:
    s = {"model.embed_tokens.weight": (g.vocab, g.hidden), "model.norm.weight": (g.hidden,),
         "cb0_head.weight": (g.n_cb0, g.hidden)}
    for i in range(g.layers):
        p = f"model.layers.{i}."
        s.update({p + "input_layernorm.weight": (g.hidden,), p + "post_attention_layernorm.weight": (g.hidden,),
                  p + "self_attn.q_proj.weight": (g.heads * g.head_dim, g.hidden),
                  p + "self_attn.k_proj.weight": (g.kv_heads * g.head_dim, g.hidden),
                  p + "self_attn.v_proj.weight": (g.kv_heads * g.head_dim, g.hidden),
                  p + "self_attn.o_proj.weight": (g.hidden, g.heads * g.head_dim),
                  p + "self_attn.q_norm.weight": (g.head_dim,), p + "self_attn.k_norm.weight": (g.head_dim,),
                  p + "mlp.gate_proj.weight": (g.ffn, g.hidden), p + "mlp.up_proj.weight": (g.ffn, g.hidden),
                  p + "mlp.down_proj.weight": (g.hidden, g.ffn)})
    return s


def depth_shapes(g: DepthGeom) -> dict:
    D = g.d
    s = {"depth.in_proj.weight": (D, g.d_backbone), "depth.code_lo.weight": ((g.n_q - 1) * g.n_codes, g.rank),
         "depth.code_up.weight": (D, g.rank), "depth.level_emb.weight": (g.n_q, D),
         "depth.norm.weight": (D,), "depth.norm.bias": (D,),
         "depth.spk_proj_ecapa.weight": (D, 192), "depth.spk_proj_campp.weight": (D, 1024),
         "depth.null_mem": (1, 1, D),
         "audio_in.table.weight": (g.n_q * g.n_codes, g.d_backbone), "audio_in.aeos_in": (g.d_backbone,),
         "audio_in.norm.weight": (g.d_backbone,)}
    for grp in range(g.n_groups):
        for li in range(g.layers):
            p = f"depth.groups.{grp}.{li}."
            s.update({p + "n1.weight": (D,), p + "n1.bias": (D,), p + "n2.weight": (D,), p + "n2.bias": (D,),
                      p + "qkv.weight": (3 * D, D), p + "o.weight": (D, D), p + "f1.weight": (g.ffn, D),
                      p + "f2.weight": (D, g.ffn)})
    for li in range(g.layers):
        p = f"depth.cross.{li}."
        s.update({p + "n.weight": (D,), p + "n.bias": (D,), p + "q.weight": (D, D), p + "kv.weight": (2 * D, D),
                  p + "o.weight": (D, D)})
    for lv in range(g.n_q - 1):
        s[f"depth.heads.{lv}.weight"] = (g.n_codes, D)
    return s


def mimi_decoder_layout(g: MimiGeom) -> list:
    """HF MimiDecoder.layers as (index, kind, c_in, c_out, kernel, stride) (transformers MimiDecoder.__init__):
    conv k7, then per ratio [ELU, ConvT(C -> C/2, 2r, r), Resnet(C/2)], then ELU and conv k3 -> 1 channel."""
    out = []
    scale = 2 ** len(g.ratios)
    out.append((0, "conv", g.hidden, scale * g.num_filters, g.kernel, 1))
    idx = 1
    for r in g.ratios:
        c = scale * g.num_filters
        out.append((idx + 1, "convt", c, c // 2, 2 * r, r))
        out.append((idx + 2, "resnet", c // 2, c // 2 // g.compress, g.res_kernel, 1))
        idx += 3
        scale //= 2
    out.append((idx + 1, "conv", g.num_filters, 1, g.last_kernel, 1))
    return out


def mimi_shapes(g: MimiGeom) -> dict:
    s = {}
    sem = "mimi.quantizer.semantic_residual_vector_quantizer."
    aco = "mimi.quantizer.acoustic_residual_vector_quantizer."
    for i in range(g.n_semantic):
        s[sem + f"layers.{i}.codebook.embed_sum"] = (g.codebook_size, g.codebook_dim)
        s[sem + f"layers.{i}.codebook.cluster_usage"] = (g.codebook_size,)
    for i in range(g.n_q - g.n_semantic):
        s[aco + f"layers.{i}.codebook.embed_sum"] = (g.codebook_size, g.codebook_dim)
        s[aco + f"layers.{i}.codebook.cluster_usage"] = (g.codebook_size,)
    s[sem + "output_proj.weight"] = (g.hidden, g.codebook_dim, 1)
    s[aco + "output_proj.weight"] = (g.hidden, g.codebook_dim, 1)
    s["mimi.upsample.conv.weight"] = (g.hidden, 1, 2 * g.upsample_stride)
    for i in range(g.layers):
        p = f"mimi.decoder_transformer.layers.{i}."
        H = g.hidden
        s.update({p + "input_layernorm.weight": (H,), p + "input_layernorm.bias": (H,),
                  p + "post_attention_layernorm.weight": (H,), p + "post_attention_layernorm.bias": (H,),
                  p + "self_attn.q_proj.weight": (H, H), p + "self_attn.k_proj.weight": (H, H),
                  p + "self_attn.v_proj.weight": (H, H), p + "self_attn.o_proj.weight": (H, H),
                  p + "mlp.fc1.weight": (g.ffn, H), p + "mlp.fc2.weight": (H, g.ffn),
                  p + "self_attn_layer_scale.scale": (H,), p + "mlp_layer_scale.scale": (H,)})
    for idx, kind, cin, cout, k, stride in mimi_decoder_layout(g):
        p = f"mimi.decoder.layers.{idx}."
        if kind == "conv":
            s[p + "conv.weight"] = (cout, cin, k)
            s[p + "conv.bias"] = (cout,)
        elif kind == "convt":
            s[p + "conv.weight"] = (cin, cout, k)
            s[p + "conv.bias"] = (cout,)
        else:
            hid = cout
            s[p + "block.1.conv.weight"] = (hid, cin, k)
            s[p + "block.1.conv.bias"] = (hid,)
            s[p + "block.3.conv.weight"] = (cin, hid, 1)
            s[p + "block.3.conv.bias"] = (cin,)
    return s


def generate(shapes: dict, seed: int = 0, device=None) -> dict:
    return {name: make(name, shape, seed, device) for name, shape in shapes.items()}


def all_shapes(geom) -> dict:
    """Every tensor the decode tick reads, for a Maya3Geom."""
    s = backbone_shapes(geom.backbone)
    s.update(depth_shapes(geom.depth))
    s.update(mimi_shapes(geom.mimi))
    return s


def backbone_weights(g: BackboneGeom, seed: int = 0) -> dict:
    return generate(backbone_shapes(g), seed)


def depth_weights(g: DepthGeom, seed: int = 0) -> dict:
    return generate(depth_shapes(g), seed)


def mimi_weights(g: MimiGeom, seed: int = 0) -> dict:
    return generate(mimi_shapes(g), seed)
