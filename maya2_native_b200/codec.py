"""StaticMimi: drop-in replacement of serve/fast_codec.py:StaticMimi on the B200 C ABI.

Same constructor, ``warmup``/``reset``/``decode``/``state_bytes_per_slot`` and ``samples_per_frame``.  Per-slot
streaming state (conv histories + transposed-conv tails as one flat channels-last row per slot, the decoder
transformer's KV ring with absolute key positions) is owned here and updated in place by ``m3_mimi_decode``; one
call per frame, replayed from a CUDA graph per batch bucket (serve/fast_codec.py:194-219).
"""
from __future__ import annotations

import math
from collections.abc import Mapping

import torch

from . import _lib as L
from .config import MimiGeom
from .weights import mimi_decoder_layout

NEVER = -(1 << 40)


def _named(mimi) -> Mapping:
    if isinstance(mimi, Mapping):
        return mimi
    return {"mimi." + k: v for k, v in mimi.state_dict().items()}


def geom_from_hf(cfg) -> MimiGeom:
    return MimiGeom(hidden=cfg.hidden_size, n_q=cfg.num_quantizers, n_semantic=cfg.num_semantic_quantizers,
                    codebook_size=cfg.codebook_size, codebook_dim=cfg.codebook_dim, layers=cfg.num_hidden_layers,
                    heads=cfg.num_attention_heads, ffn=cfg.intermediate_size, window=cfg.sliding_window,
                    ratios=tuple(cfg.upsampling_ratios), num_filters=cfg.num_filters, kernel=cfg.kernel_size,
                    last_kernel=cfg.last_kernel_size, res_kernel=cfg.residual_kernel_size, compress=cfg.compress,
                    rope_theta=(cfg.rope_parameters or {}).get("rope_theta", 1e4), norm_eps=cfg.norm_eps)


class _Bucket:
    __slots__ = ("graph", "slots", "codes", "out", "pinned", "events", "turn")


class StaticMimi:
    def __init__(self, mimi, max_slots, batch_buckets=(1, 2, 4, 8, 16, 24, 32, 48, 64, 80, 96), ring=256,
                 geom: MimiGeom | None = None, device=None):
        sd = _named(mimi)
        if geom is None:
            geom = geom_from_hf(mimi.config)
        g = geom if geom.ring == ring else MimiGeom(**{**geom.__dict__, "ring": int(ring)})
        if g.ring < g.window + g.upsample_stride:
            raise ValueError("ring must hold sliding_window + frame_tokens entries")
        self.geom = g
        self.device = torch.device(device) if device is not None else torch.device("cuda", torch.cuda.current_device())
        self.dtype = torch.bfloat16
        self.max_slots, self.dummy = int(max_slots), int(max_slots)
        self.batch_buckets = tuple(sorted(set(int(b) for b in batch_buckets)))
        self.window, self.ring, self.frame_tokens = g.window, g.ring, g.upsample_stride
        self.codebooks = g.n_q
        self.kv_heads, self.head_dim = g.heads, g.head_dim
        dev, bf = self.device, self.dtype

        def w(name):
            return sd["mimi." + name].detach().to(dev, bf).contiguous()
        with torch.inference_mode():
            sem = "quantizer.semantic_residual_vector_quantizer."
            aco = "quantizer.acoustic_residual_vector_quantizer."
            books = []
            for i in range(g.n_q):
                p = f"{sem}layers.{i}." if i < g.n_semantic else f"{aco}layers.{i - g.n_semantic}."
                # MimiEuclideanCodebook.embed in the model dtype: embed_sum / cluster_usage.clamp(min=1e-5)
                books.append(w(p + "codebook.embed_sum") / w(p + "codebook.cluster_usage").clamp(min=1e-5)[:, None])
            self.books = torch.stack(books).contiguous()
            self.proj_sem = w(sem + "output_proj.weight")[:, :, 0].contiguous()
            self.proj_ac = w(aco + "output_proj.weight")[:, :, 0].contiguous()
            self.upw = w("upsample.conv.weight")[:, 0, :].contiguous()
            self._t = {k: [] for k in ("ln1_w", "ln1_b", "wqkv", "wo", "ln2_w", "ln2_b", "fc1", "fc2", "ls1", "ls2")}
            for i in range(g.layers):
                p = f"decoder_transformer.layers.{i}."
                a = p + "self_attn."
                self._t["ln1_w"].append(w(p + "input_layernorm.weight"))
                self._t["ln1_b"].append(w(p + "input_layernorm.bias"))
                self._t["wqkv"].append(torch.cat([w(a + "q_proj.weight"), w(a + "k_proj.weight"),
                                                  w(a + "v_proj.weight")]).contiguous())
                self._t["wo"].append(w(a + "o_proj.weight"))
                self._t["ln2_w"].append(w(p + "post_attention_layernorm.weight"))
                self._t["ln2_b"].append(w(p + "post_attention_layernorm.bias"))
                self._t["fc1"].append(w(p + "mlp.fc1.weight"))
                self._t["fc2"].append(w(p + "mlp.fc2.weight"))
                self._t["ls1"].append(w(p + "self_attn_layer_scale.scale"))
                self._t["ls2"].append(w(p + "mlp_layer_scale.scale"))
            hd = g.head_dim
            inv = 1.0 / (g.rope_theta ** (torch.arange(0, hd, 2, dtype=torch.int64).float() / hd))
            self.inv_freq = inv.to(bf).float().to(dev).contiguous()   # the model's buffer, in the model dtype
            self._s = {k: [] for k in ("convt_w", "convt_b", "res1_w", "res1_b", "res2_w", "res2_b")}

            def conv_pack(t):  # [c_out, c_in, k] -> [c_out, k * c_in], element (o, j*c_in + i) = W[o, i, j]
                return t.permute(0, 2, 1).reshape(t.shape[0], -1).contiguous()
            for idx, kind, cin, cout, k, stride in mimi_decoder_layout(g):
                p = f"decoder.layers.{idx}."
                if kind == "conv" and idx == 0:
                    self.conv0_w, self.conv0_b = conv_pack(w(p + "conv.weight")), w(p + "conv.bias")
                elif kind == "conv":
                    self.final_w, self.final_b = conv_pack(w(p + "conv.weight")), w(p + "conv.bias")
                elif kind == "convt":  # [c_in, c_out, 2r] -> [2r * c_out, c_in], element (j*c_out + o, i) = W[i, o, j]
                    t = w(p + "conv.weight")
                    self._s["convt_w"].append(t.permute(2, 1, 0).reshape(-1, t.shape[0]).contiguous())
                    self._s["convt_b"].append(w(p + "conv.bias"))
                else:
                    self._s["res1_w"].append(conv_pack(w(p + "block.1.conv.weight")))
                    self._s["res1_b"].append(w(p + "block.1.conv.bias"))
                    self._s["res2_w"].append(conv_pack(w(p + "block.3.conv.weight")))
                    self._s["res2_b"].append(w(p + "block.3.conv.bias"))
            rows = self.max_slots + 1
            self._cfg = L.MimiConfig(g.hidden, g.n_q, g.n_semantic, g.codebook_size, g.codebook_dim, g.layers,
                                     g.heads, g.ffn, g.window, g.ring, len(g.ratios),
                                     (L.i32 * 8)(*(list(g.ratios) + [0] * (8 - len(g.ratios)))), g.num_filters,
                                     g.kernel, g.last_kernel, g.res_kernel, g.compress, g.upsample_stride,
                                     self.max_slots, max(self.batch_buckets), g.norm_eps)
            elems = int(L.load().m3_mimi_state_elems(self._cfg))
            self.conv_flat = torch.zeros(rows, elems, device=dev, dtype=bf)
            self.kv = torch.zeros(g.layers, 2, rows, g.heads, g.ring, g.head_dim, device=dev, dtype=bf)
            self.key_pos = torch.full((rows, g.ring), NEVER, device=dev, dtype=torch.long)
            self.tokens = torch.zeros(rows, device=dev, dtype=torch.long)
        self.samples_per_frame = g.samples_per_frame
        self._buckets = {}
        self._pool = None
        self._handle = self._create()

    def _create(self):
        t = {k: L.ptr_array([x.data_ptr() for x in v]) for k, v in self._t.items()}
        s = {k: L.ptr_array([x.data_ptr() for x in v]) for k, v in self._s.items()}
        self._keep = (t, s)
        wts = L.MimiWeights(self.books.data_ptr(), self.proj_sem.data_ptr(), self.proj_ac.data_ptr(),
                            self.upw.data_ptr(), t["ln1_w"], t["ln1_b"], t["wqkv"], t["wo"], t["ln2_w"], t["ln2_b"],
                            t["fc1"], t["fc2"], t["ls1"], t["ls2"], self.inv_freq.data_ptr(), self.conv0_w.data_ptr(),
                            self.conv0_b.data_ptr(), s["convt_w"], s["convt_b"], s["res1_w"], s["res1_b"],
                            s["res2_w"], s["res2_b"], self.final_w.data_ptr(), self.final_b.data_ptr(),
                            self.conv_flat.data_ptr(), self.kv.data_ptr(), self.key_pos.data_ptr(),
                            self.tokens.data_ptr())
        h = L.vp()
        L.check(L.load().m3_mimi_create(self._cfg, wts, h), "m3_mimi_create")
        return h

    def close(self):
        if getattr(self, "_handle", None):
            self._buckets.clear()
            L.load().m3_mimi_destroy(self._handle)
            self._handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def device_status(self, clear=True) -> int:
        s = L.i32(0)
        L.check(L.load().m3_mimi_status(self._handle, s, int(clear)), "m3_mimi_status")
        return int(s.value)

    def set_sm_budget(self, sms: int):
        """SMs the persistent SEANet kernels spread over (0: all); for a decoder on a second stream beside other
        work.  Graphs captured afterwards use it; results do not depend on it."""
        L.check(L.load().m3_mimi_set_sm_budget(self._handle, int(sms)), "m3_mimi_set_sm_budget")

    def state_bytes_per_slot(self):
        return {"conv": self.conv_flat[0].numel() * self.conv_flat.element_size(),
                "attention_kv": self.kv[:, :, 0].numel() * self.kv.element_size(),
                "attention_index": self.key_pos[0].numel() * 8 + 8}

    def _reset_row(self, row, zero_kv=False):
        L.check(L.load().m3_mimi_reset(self._handle, int(row), int(zero_kv), L.stream_ptr()), "m3_mimi_reset")

    @torch.inference_mode()
    def reset(self, slot, zero_kv=False):
        """serve/fast_codec.py:236-244: clear the slot's conv state, ring positions and token count."""
        if not 0 <= slot < self.max_slots:
            raise IndexError(f"slot {slot} outside [0,{self.max_slots})")
        self._reset_row(slot, zero_kv)

    def _launch(self, b, stream=None):
        L.check(L.load().m3_mimi_decode(self._handle, b.slots.data_ptr(), b.codes.data_ptr(), b.out.data_ptr(),
                                        b.slots.shape[0], L.stream_ptr(stream)), "m3_mimi_decode")

    @torch.inference_mode()
    def _capture(self, size):
        dev = self.device
        b = _Bucket()
        b.slots = torch.full((size,), self.dummy, device=dev, dtype=torch.long)
        b.codes = torch.zeros(size, self.codebooks, device=dev, dtype=torch.long)
        b.out = torch.zeros(size, self.samples_per_frame, device=dev, dtype=torch.float32)
        b.pinned = [torch.full((size,), self.dummy, dtype=torch.long).pin_memory() for _ in range(8)]
        b.events = [None] * len(b.pinned)
        b.turn = 0
        side = torch.cuda.Stream(device=dev)
        side.wait_stream(torch.cuda.current_stream(dev))
        with torch.cuda.stream(side):
            for _ in range(2):   # only the dummy slot is touched
                self._launch(b, side)
        torch.cuda.current_stream(dev).wait_stream(side)
        torch.cuda.synchronize(dev)
        if self._pool is None:
            self._pool = torch.cuda.graph_pool_handle()
        b.graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(b.graph, pool=self._pool):
            self._launch(b)
        self._reset_row(self.dummy)
        self._buckets[size] = b
        return b

    @torch.inference_mode()
    def warmup(self, batch_buckets=None):
        sizes = self.batch_buckets if batch_buckets is None else tuple(sorted(set(int(b) for b in batch_buckets)))
        for size in sorted(sizes, reverse=True):
            if size not in self._buckets:
                self._capture(size)
        self.batch_buckets = tuple(sorted(set(self.batch_buckets) | set(sizes)))

    @torch.inference_mode()
    def decode(self, slots, codes):
        """serve/fast_codec.py:246-277: codes [B, K] long -> owned fp32 PCM [B, samples_per_frame]."""
        count = len(slots)
        if codes.shape[0] != count or codes.dim() != 2 or codes.shape[1] != self.codebooks:
            raise ValueError(f"codes must be [{count},{self.codebooks}], got {tuple(codes.shape)}")
        size = next((b for b in self.batch_buckets if b >= count), None)
        if size is None:
            raise ValueError(f"batch {count} exceeds largest bucket {self.batch_buckets[-1]}")
        b = self._buckets.get(size) or self._capture(size)
        if torch.is_tensor(slots):
            b.slots[:count].copy_(slots)
            b.slots[count:].fill_(self.dummy)
        else:
            if len(set(slots)) != count or min(slots) < 0 or max(slots) >= self.max_slots:
                raise ValueError("slots must be distinct and inside [0,max_slots)")
            turn = b.turn
            b.turn = (turn + 1) % len(b.pinned)
            if b.events[turn] is not None:
                b.events[turn].synchronize()
            staging = b.pinned[turn]
            staging[:count] = torch.tensor(slots, dtype=torch.long)
            staging[count:] = self.dummy
            b.slots.copy_(staging, non_blocking=True)
            ev = torch.cuda.Event()
            ev.record()
            b.events[turn] = ev
        b.codes[:count].copy_(codes)
        b.graph.replay()
        return b.out[:count].clone()


def sample_rate_ok(g: MimiGeom) -> bool:
    return math.prod(g.ratios) * g.upsample_stride == g.samples_per_frame
