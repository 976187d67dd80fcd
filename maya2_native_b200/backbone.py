"""StaticBackbone: drop-in replacement of serve/fast_backbone.py:StaticBackbone on the B200 C ABI.

Same constructor, methods and engine-visible attributes (``lengths``, ``lengths_cpu``, ``kv_heads``, ``head_dim``,
``layers``, ``k``/``v`` per-layer caches).  One decode path only: the ``attention``/``fuse_*``/``fused_norm``
switches are accepted for signature compatibility and do not select anything (the reference's own validation of
``attention`` is kept).  Each step is one ``m3_backbone_step`` call, replayed from a CUDA graph per
(row bucket, context bucket) exactly like the reference's graph cache (serve/fast_backbone.py:249-315).
"""
from __future__ import annotations

from collections.abc import Mapping

import numpy as np
import torch

from . import _lib as L


def state_dict_of(source) -> Mapping:
    """Named tensors of a backbone source: a mapping of HF Qwen3 names ('model.layers.0...'), an HF causal LM, or
    the reference's Backbone wrapper (its ``.lm``)."""
    if isinstance(source, Mapping):
        return source
    lm = getattr(source, "lm", source)
    return lm.state_dict()


def rope_tables(head_dim: int, capacity: int, theta: float, dtype: torch.dtype):
    """Qwen3 default RoPE tables [capacity, head_dim] in the model dtype.  The reference computes them with the
    model's own rotary module after the model was cast to its serving dtype (tts/model/load_s3.py:417-419), so the
    inverse frequencies are rounded to that dtype first (serve/fast_backbone.py:151-153)."""
    inv = 1.0 / (theta ** (torch.arange(0, head_dim, 2, dtype=torch.int64).float() / head_dim))
    inv = inv.to(dtype).float()
    f = torch.arange(capacity, dtype=torch.float32)[:, None] * inv[None, :]
    emb = torch.cat([f, f], -1)
    return emb.cos().to(dtype), emb.sin().to(dtype)


class _Graph:
    __slots__ = ("graph", "slots", "slots_cpu", "x", "real", "real_cpu", "out", "last", "offset", "offset_cpu",
                 "offset_dirty", "evt")


class StaticBackbone:
    def __init__(self, backbone, max_slots, capacity=1536, batch_buckets=(1, 2, 4, 8, 16, 24, 32, 48, 64, 80, 96),
                 ctx_buckets=(512, 768, 1024, 1536), attention="gather", fused_norm=False, use_graphs=True,
                 fuse_proj=False, fuse_rope=False, geom=None, device=None):
        if attention not in ("gather", "triton"):
            raise ValueError("attention must be gather or triton")
        sd = state_dict_of(backbone)
        cfg = getattr(getattr(backbone, "lm", backbone), "config", None)
        if geom is None:
            if cfg is None:
                raise ValueError("pass geom= when the backbone source is a plain mapping")
            from .config import BackboneGeom
            geom = BackboneGeom(layers=cfg.num_hidden_layers, hidden=cfg.hidden_size, heads=cfg.num_attention_heads,
                                kv_heads=cfg.num_key_value_heads,
                                head_dim=getattr(cfg, "head_dim", cfg.hidden_size // cfg.num_attention_heads),
                                ffn=cfg.intermediate_size, vocab=cfg.vocab_size, eps=cfg.rms_norm_eps,
                                rope_theta=(getattr(cfg, "rope_parameters", None) or {}).get("rope_theta", 1e6))
        self.geom = g = geom
        self.device = torch.device(device) if device is not None else torch.device("cuda", torch.cuda.current_device())
        self.dtype = torch.bfloat16
        self.heads, self.kv_heads, self.head_dim = g.heads, g.kv_heads, g.head_dim
        self.groups, self.hidden = g.heads // g.kv_heads, g.hidden
        self.scaling, self.eps = g.head_dim ** -0.5, g.eps
        self.max_slots, self.capacity, self.dummy = int(max_slots), int(capacity), int(max_slots)
        self.attention, self.fused_norm, self.use_graphs = attention, fused_norm, use_graphs
        self.layers = list(range(g.layers))
        self.batch_buckets = tuple(sorted(set(int(b) for b in batch_buckets)))
        if self.batch_buckets[-1] < self.max_slots:
            self.batch_buckets += (self.max_slots,)
        self.ctx_buckets = tuple(sorted({min(int(c), self.capacity) for c in ctx_buckets} | {self.capacity}))
        dev, bf = self.device, self.dtype

        def w(name):
            return sd[name].detach().to(device=dev, dtype=bf).contiguous()
        with torch.inference_mode():
            self._w = {"in_norm": [], "wqkv": [], "q_norm": [], "k_norm": [], "wo": [], "post_norm": [], "wgu": [],
                       "wdown": []}
            for i in range(g.layers):
                p = f"model.layers.{i}."
                self._w["in_norm"].append(w(p + "input_layernorm.weight"))
                self._w["wqkv"].append(torch.cat([w(p + "self_attn.q_proj.weight"), w(p + "self_attn.k_proj.weight"),
                                                  w(p + "self_attn.v_proj.weight")]).contiguous())
                self._w["q_norm"].append(w(p + "self_attn.q_norm.weight"))
                self._w["k_norm"].append(w(p + "self_attn.k_norm.weight"))
                self._w["wo"].append(w(p + "self_attn.o_proj.weight"))
                self._w["post_norm"].append(w(p + "post_attention_layernorm.weight"))
                self._w["wgu"].append(torch.cat([w(p + "mlp.gate_proj.weight"), w(p + "mlp.up_proj.weight")])
                                      .contiguous())
                self._w["wdown"].append(w(p + "mlp.down_proj.weight"))
            self.final_norm = w("model.norm.weight")
            cos, sin = rope_tables(g.head_dim, self.capacity, g.rope_theta, bf)
            self.cos, self.sin = cos.to(dev).contiguous(), sin.to(dev).contiguous()
            shape = (self.max_slots + 1, g.kv_heads, self.capacity, g.head_dim)
            self.k = [torch.zeros(shape, dtype=bf, device=dev) for _ in range(g.layers)]
            self.v = [torch.zeros(shape, dtype=bf, device=dev) for _ in range(g.layers)]
            self.lengths = torch.zeros(self.max_slots + 1, dtype=torch.long, device=dev)
            self.lengths_cpu = [0] * (self.max_slots + 1)
        self.graphs = {}
        self.pool = None
        self.max_rows = max(self.batch_buckets)
        self._handle = self._create()

    # ---------------------------------------------------------------- native handle
    def _create(self):
        lib = L.load()
        g = self.geom
        cfg = L.BackboneConfig(g.layers, g.hidden, g.heads, g.kv_heads, g.head_dim, g.ffn, self.max_slots,
                               self.capacity, self.max_rows, g.eps)
        arrs = {k: L.ptr_array([t.data_ptr() for t in v]) for k, v in self._w.items()}
        self._keep = arrs
        kc = L.ptr_array([t.data_ptr() for t in self.k])
        vc = L.ptr_array([t.data_ptr() for t in self.v])
        self._keep_kv = (kc, vc)
        wts = L.BackboneWeights(arrs["in_norm"], arrs["wqkv"], arrs["q_norm"], arrs["k_norm"], arrs["wo"],
                                arrs["post_norm"], arrs["wgu"], arrs["wdown"], self.final_norm.data_ptr(),
                                self.cos.data_ptr(), self.sin.data_ptr(), kc, vc, self.lengths.data_ptr())
        h = L.vp()
        L.check(lib.m3_backbone_create(cfg, wts, h), "m3_backbone_create")
        return h

    def close(self):
        if getattr(self, "_handle", None):
            self.graphs.clear()
            L.load().m3_backbone_destroy(self._handle)
            self._handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def device_status(self, clear=True) -> int:
        s = L.i32(0)
        L.check(L.load().m3_backbone_status(self._handle, s, int(clear)), "m3_backbone_status")
        return int(s.value)

    # ---------------------------------------------------------------- slots
    @torch.inference_mode()
    def load_slot(self, slot, hf_cache, length):
        """serve/fast_backbone.py:157-165: install an HF DynamicCache's first `length` positions into a slot."""
        if not 0 <= slot < self.max_slots:
            raise IndexError(slot)
        if length > self.capacity:
            raise ValueError(f"length {length} exceeds capacity {self.capacity}")
        for i in self.layers:
            layer = hf_cache.layers[i]
            self.k[i][slot, :, :length].copy_(layer.keys[0, :, :length])
            self.v[i][slot, :, :length].copy_(layer.values[0, :, :length])
        self.lengths[slot] = length
        self.lengths_cpu[slot] = length

    @torch.inference_mode()
    def load_prefix(self, slot, kv, length):
        """serve/fast_backbone.py:317-323: install a stored prefix KV (per-layer (k, v) [1, KV, length, D])."""
        if not 0 <= slot < self.max_slots:
            raise IndexError(slot)
        for i, (k, v) in enumerate(kv):
            self.k[i][slot, :, :length].copy_(k[0])
            self.v[i][slot, :, :length].copy_(v[0])
        self.lengths[slot] = length
        self.lengths_cpu[slot] = length

    # ---------------------------------------------------------------- voice prefixes (packed store, one launch)
    def prefix_store(self, length) -> torch.Tensor:
        """An empty packed prefix store bf16 [layers, 2 (K, V), kv_heads, length, head_dim] (m3_backbone_*_prefix)."""
        g = self.geom
        return torch.empty(g.layers, 2, g.kv_heads, int(length), g.head_dim, dtype=torch.bfloat16, device=self.device)

    def _check_store(self, store, length):
        g = self.geom
        if tuple(store.shape) != (g.layers, 2, g.kv_heads, int(length), g.head_dim) or store.dtype != torch.bfloat16 \
                or store.device != self.device or not store.is_contiguous():
            raise ValueError("prefix store must be contiguous bf16 [layers, 2, kv_heads, length, head_dim] on the "
                             "backbone's device")

    @torch.inference_mode()
    def save_prefix(self, slot, length, store=None) -> torch.Tensor:
        """The slot's first `length` positions of every layer's K/V as a packed store (one launch)."""
        if not 0 <= slot < self.max_slots:
            raise IndexError(slot)
        if not 0 < length <= self.lengths_cpu[slot]:
            raise ValueError(f"slot {slot} holds {self.lengths_cpu[slot]} positions, asked for {length}")
        store = self.prefix_store(length) if store is None else store
        self._check_store(store, length)
        L.check(L.load().m3_backbone_save_prefix(self._handle, slot, store.data_ptr(), int(length), L.stream_ptr()),
                "m3_backbone_save_prefix")
        return store

    @torch.inference_mode()
    def load_prefix_store(self, slot, store, length):
        """load_prefix from a packed store (serve/fast_backbone.py:316-322 in one launch): K/V rows [0, length) of the
        slot and its length (device and host mirror)."""
        if not 0 <= slot < self.max_slots:
            raise IndexError(slot)
        if not 0 < length <= self.capacity:
            raise ValueError(f"length {length} outside (0, {self.capacity}]")
        self._check_store(store, length)
        L.check(L.load().m3_backbone_load_prefix(self._handle, slot, store.data_ptr(), int(length), L.stream_ptr()),
                "m3_backbone_load_prefix")
        self.lengths_cpu[slot] = int(length)

    @torch.inference_mode()
    def build_prefix(self, slot, x, chunk=None) -> torch.Tensor:
        """A voice's prefix KV computed by this backbone (maya3/engine.py:276-280 runs an eager HF prefill for it): the
        prefix embeddings x [T, hidden] are prefilled into the free `slot` by inline-prefill steps of at most `chunk`
        rows, saved as a packed store, and the slot is freed again."""
        T = int(x.shape[0])
        chunk = int(chunk or self.max_rows)
        self.free(slot)
        for c0 in range(0, T, chunk):
            self.step_mixed([], None, [(slot, x[c0:c0 + chunk])])
        store = self.save_prefix(slot, T)
        self.free(slot)
        return store

    @torch.inference_mode()
    def free(self, slot):
        self.lengths[slot] = 0
        self.lengths_cpu[slot] = 0

    def memory_bytes(self):
        return sum(t.numel() * t.element_size() for t in self.k + self.v)

    # ---------------------------------------------------------------- graphs
    def _bucket(self, values, need, what):
        for b in values:
            if b >= need:
                return b
        raise ValueError(f"{what} {need} exceeds largest bucket {values[-1]}")

    def _launch(self, g, cb, stream=None):
        L.check(L.load().m3_backbone_step(self._handle, g.slots.data_ptr(), g.offset.data_ptr(), g.real.data_ptr(),
                                          g.x.data_ptr(), g.out.data_ptr(), g.slots.shape[0], cb,
                                          L.stream_ptr(stream)), "m3_backbone_step")

    @torch.inference_mode()
    def _capture(self, bb, cb):
        dev = self.device
        g = _Graph()
        g.slots = torch.full((bb,), self.dummy, dtype=torch.long, device=dev)
        g.real = torch.zeros(bb, dtype=torch.long, device=dev)
        g.offset = torch.zeros(bb, dtype=torch.long, device=dev)
        g.offset_cpu = torch.zeros(bb, dtype=torch.long).pin_memory()
        g.offset_dirty = False
        g.x = torch.zeros(bb, self.hidden, dtype=self.dtype, device=dev)
        g.out = torch.zeros(bb, self.hidden, dtype=self.dtype, device=dev)
        g.slots_cpu = torch.full((bb,), self.dummy, dtype=torch.long).pin_memory()
        g.real_cpu = torch.zeros(bb, dtype=torch.long).pin_memory()
        g.last = None
        g.graph = None
        g.evt = None
        if self.use_graphs:
            stream = torch.cuda.Stream()
            stream.wait_stream(torch.cuda.current_stream())
            with torch.cuda.stream(stream):
                for _ in range(2):   # all-dummy rows: touches only the dummy slot (lazy library init happens here)
                    self._launch(g, cb, stream)
            torch.cuda.current_stream().wait_stream(stream)
            if self.pool is None:
                self.pool = torch.cuda.graph_pool_handle()
            g.graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g.graph, pool=self.pool):
                self._launch(g, cb)
        self.graphs[bb, cb] = g
        return g

    @torch.inference_mode()
    def warmup(self, batch_buckets=None, ctx_buckets=None):
        for bb in sorted(batch_buckets or self.batch_buckets, reverse=True):
            for cb in sorted(ctx_buckets or self.ctx_buckets, reverse=True):
                cb = min(cb, self.capacity)
                if (bb, cb) not in self.graphs:
                    self._capture(bb, cb)
        torch.cuda.synchronize()

    def _run(self, g, cb):
        if g.graph is not None:
            g.graph.replay()
        else:
            self._launch(g, cb)

    @torch.inference_mode()
    def step(self, slots, x):
        """serve/fast_backbone.py:288-315: one decode row per distinct slot -> owned [B, hidden]."""
        B = len(slots)
        if B == 0:
            return x.new_zeros(0, self.hidden)
        if len(set(slots)) != B:
            raise ValueError("duplicate slots in one step")
        need = 0
        for s in slots:
            if not 0 <= s < self.max_slots:
                raise IndexError(s)
            need = max(need, self.lengths_cpu[s] + 1)
        if need > self.capacity:
            raise ValueError(f"context {need} exceeds capacity {self.capacity}")
        bb = self._bucket(self.batch_buckets, B, "batch")
        cb = self._bucket(self.ctx_buckets, need, "context")
        g = self.graphs.get((bb, cb)) or self._capture(bb, cb)
        key = tuple(slots)
        if g.offset_dirty:
            g.offset.zero_()
            g.offset_dirty = False
            g.last = None
        if g.last != key:
            if g.evt is not None:
                g.evt.synchronize()    # pinned staging may still feed an earlier async copy
            g.slots_cpu[:B] = torch.tensor(slots, dtype=torch.long)
            g.slots_cpu[B:] = self.dummy
            g.real_cpu[:B] = 1
            g.real_cpu[B:] = 0
            g.slots.copy_(g.slots_cpu, non_blocking=True)
            g.real.copy_(g.real_cpu, non_blocking=True)
            g.evt = torch.cuda.Event()
            g.evt.record()
            g.last = key
        g.x[:B].copy_(x)
        self._run(g, cb)
        out = g.out[:B].clone()
        for s in slots:
            self.lengths_cpu[s] += 1
        return out

    @torch.inference_mode()
    def step_mixed(self, slots, x, prefills):
        """serve/fast_backbone.py:325-359: decode rows plus inline prefills (slot, x_tokens [T, hidden]), each
        prefill contributing T rows of its slot at consecutive positions.  Returns (decoded [B, hidden],
        [last hidden per prefill])."""
        B = len(slots)
        rows = B + sum(t.shape[0] for _, t in prefills)
        if rows == 0:
            return (x.new_zeros(0, self.hidden) if x is not None else
                    torch.zeros(0, self.hidden, dtype=self.dtype, device=self.device)), []
        if len(set(slots) | {s for s, _ in prefills}) != B + len(prefills):
            raise ValueError("duplicate slots in one step")
        for s in list(slots) + [s for s, _ in prefills]:
            if not 0 <= s < self.max_slots:
                raise IndexError(s)
        need = max([self.lengths_cpu[s] + 1 for s in slots] + [self.lengths_cpu[s] + t.shape[0] for s, t in prefills])
        if need > self.capacity:
            raise ValueError(f"context {need} exceeds capacity {self.capacity}")
        bb = self._bucket(self.batch_buckets, rows, "batch")
        cb = self._bucket(self.ctx_buckets, need, "context")
        g = self.graphs.get((bb, cb)) or self._capture(bb, cb)
        if g.evt is not None:
            g.evt.synchronize()
        index = list(slots)
        offsets = [0] * B
        for s, t in prefills:
            index += [s] * t.shape[0]
            offsets += range(t.shape[0])
        g.slots_cpu[:rows] = torch.tensor(index, dtype=torch.long)
        g.slots_cpu[rows:] = self.dummy
        g.offset_cpu[:rows] = torch.tensor(offsets, dtype=torch.long)
        g.offset_cpu[rows:] = 0
        g.real_cpu[:rows] = 1
        g.real_cpu[rows:] = 0
        g.slots.copy_(g.slots_cpu, non_blocking=True)
        g.real.copy_(g.real_cpu, non_blocking=True)
        g.offset.copy_(g.offset_cpu, non_blocking=True)
        g.last = None
        g.offset_dirty = bool(prefills)
        g.evt = torch.cuda.Event()
        g.evt.record()
        if B:
            g.x[:B].copy_(x)
        at = B
        for _, t in prefills:
            g.x[at:at + t.shape[0]].copy_(t)
            at += t.shape[0]
        self._run(g, cb)
        out = g.out
        decoded = out[:B].clone()
        last = []
        at = B
        for s, t in prefills:
            at += t.shape[0]
            last.append(out[at - 1].clone())
            self.lengths_cpu[s] += t.shape[0]
        for s in slots:
            self.lengths_cpu[s] += 1
        return decoded, last
