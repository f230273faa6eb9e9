"""Gemma-4 decoder (decode step) over libfmoe: host-side mirror of src/model.

    Gemma4DecoderLayer.forward(x, cache, pos)   DecoderLayer::forward_gemma4, src/model/mod.rs:67-119
    Gemma4Model.decode_step(ids)                TextModel::forward + Model::forward, src/model/mod.rs:135-363
                                                (embedding, 30 layers, final norm, tied lm_head, softcap)

Two execution paths, both capturable in one CUDA graph with the decode
position kept on the device:
  decode_step        one library call per layer (fmoe_decoder_layer_forward:
                     11 kernels chained on the stream), any batch 1..8; with an
                     EPComm the layers hold expert slices and the routed experts
                     run on their owning GPUs (fmoe_decoder_layer_forward_ep);
  decode_step_fused  the whole step as one persistent kernel
                     (fmoe_decode_step), batch 1.
"""
from __future__ import annotations

import ctypes
import math
import os

import torch

from . import (ExpertTable, ExpertsC, KvCacheC, QuantizedLinear, QWeightC, RouterC, _ptr, _stream, check, lib,
               prefill_prep)
from .kv import KV_AFFINE, KV_BF16, KVCache


class DecoderLayerC(ctypes.Structure):
    _fields_ = [
        ("q_proj", QWeightC), ("k_proj", QWeightC), ("v_proj", QWeightC), ("o_proj", QWeightC),
        ("q_norm", ctypes.c_void_p), ("k_norm", ctypes.c_void_p), ("input_norm", ctypes.c_void_p),
        ("post_attn_norm", ctypes.c_void_p), ("pre_ff_norm", ctypes.c_void_p), ("post_ff_norm_1", ctypes.c_void_p),
        ("pre_ff_norm_2", ctypes.c_void_p), ("post_ff_norm_2", ctypes.c_void_p), ("post_ff_norm", ctypes.c_void_p),
        ("mlp_gate", QWeightC), ("mlp_up", QWeightC), ("mlp_down", QWeightC),
        ("router", RouterC), ("experts", ExpertsC),
        ("num_heads", ctypes.c_int32), ("num_kv_heads", ctypes.c_int32), ("head_dim", ctypes.c_int32),
        ("rope_dims", ctypes.c_int32), ("k_eq_v", ctypes.c_int32), ("sparse_v_tau", ctypes.c_float),
        ("rope_theta", ctypes.c_float), ("eps", ctypes.c_float), ("layer_scalar", ctypes.c_float),
        ("attn_scale", ctypes.c_float),
    ]


class DecodeModelC(ctypes.Structure):
    _fields_ = [
        ("n_layers", ctypes.c_int32), ("reserved", ctypes.c_int32),
        ("layers", ctypes.POINTER(DecoderLayerC)), ("caches", ctypes.POINTER(KvCacheC)),
        ("embed", QWeightC), ("final_norm", ctypes.c_void_p),
        ("eps", ctypes.c_float), ("softcap", ctypes.c_float), ("embed_scale", ctypes.c_float),
    ]


# Gemma-4 26B-A4B shapes (the reference's CLAUDE.md model notes): 30 layers,
# every fifth one full attention (head_dim 512, 2 KV heads, K == V, theta 1e6)
# and the rest sliding-window (head_dim 256, 8 KV heads, theta 1e4, window 1024).
GEMMA4_26B = dict(hidden=2816, layers=30, heads=16, sliding_kv_heads=8, sliding_head_dim=256, full_kv_heads=2,
                  full_head_dim=512, sliding_theta=1e4, full_theta=1e6, full_partial_rotary=0.25, window=1024,
                  dense_inter=2112, experts=128, expert_inter=704, top_k=8, vocab=262144, eps=1e-6, softcap=30.0,
                  attn_bits=8, dense_bits=4, embed_bits=6, router_bits=16, full_every=5)


def layer_is_full(cfg, i):
    return (i + 1) % cfg["full_every"] == 0


class Gemma4DecoderLayer:
    """Weights and hyper-parameters of one decoder layer (src/model/mod.rs:40-58,
    gemma4_attention.rs:16-33, mlp.rs:28-33, moe.rs:298-312)."""

    def __init__(self, q_proj, k_proj, v_proj, o_proj, q_norm, k_norm, norms, mlp, router, experts, num_heads,
                 num_kv_heads, head_dim, rope_dims, rope_theta, k_eq_v, eps=1e-6, layer_scalar=1.0, attn_scale=1.0,
                 top_k=8):
        self.q_proj, self.k_proj, self.v_proj, self.o_proj = q_proj, k_proj, v_proj, o_proj
        self.q_norm, self.k_norm = q_norm, k_norm
        self.norms = norms  # dict: input, post_attn, pre_ff, post_ff_1, pre_ff_2, post_ff_2, post_ff
        self.mlp = mlp      # (gate, up, down) QuantizedLinear
        self.router = router  # dict: proj QuantizedLinear, router_scale, per_expert_scale, root_size[, logit_bias]
        self.experts = experts
        self.num_heads, self.num_kv_heads, self.head_dim = num_heads, num_kv_heads, head_dim
        self.rope_dims, self.rope_theta, self.k_eq_v = rope_dims, rope_theta, k_eq_v
        self.eps, self.layer_scalar, self.attn_scale, self.top_k = eps, layer_scalar, attn_scale, top_k
        self.sparse_v_tau = 0.0  # decode-only sparse-V gate (gemma4_attention.rs:91-93); 0: off
        self._c = None

    def cstruct(self) -> DecoderLayerC:
        if self._c is None:
            n = self.norms
            empty = QWeightC(None, None, None, 0, 0, 0, 0, None, 0, 0)
            r = self.router
            rc = RouterC(r["proj"].cstruct(), _ptr(r.get("router_scale")), _ptr(r.get("per_expert_scale")),
                         _ptr(r.get("logit_bias")), r["root_size"], self.eps, 1, self.top_k)
            self._c = DecoderLayerC(
                self.q_proj.cstruct(), self.k_proj.cstruct(),
                empty if self.k_eq_v else self.v_proj.cstruct(), self.o_proj.cstruct(),
                _ptr(self.q_norm), _ptr(self.k_norm), _ptr(n["input"]), _ptr(n["post_attn"]), _ptr(n["pre_ff"]),
                _ptr(n["post_ff_1"]), _ptr(n["pre_ff_2"]), _ptr(n["post_ff_2"]), _ptr(n["post_ff"]),
                self.mlp[0].cstruct(), self.mlp[1].cstruct(), self.mlp[2].cstruct(), rc, self.experts.cstruct(),
                self.num_heads, self.num_kv_heads, self.head_dim, self.rope_dims, int(self.k_eq_v),
                float(self.sparse_v_tau), self.rope_theta, self.eps, self.layer_scalar, self.attn_scale)
        return self._c

    def tile_weights(self):
        """Tile-layout copies of the projections for the decode GEMVs (one GEMV
        launch each: q|k|v, o, dense gate|up, dense down)."""
        qkv = [self.q_proj, self.k_proj] + ([] if self.k_eq_v else [self.v_proj])
        rows = sum(q.out_features for q in qkv)
        for q in qkv:
            q.tile(rows, accumulate=False)
        self.o_proj.tile(accumulate=True)
        g, u, d = self.mlp
        g.tile(g.out_features + u.out_features, accumulate=True)
        u.tile(g.out_features + u.out_features, accumulate=True)
        d.tile(accumulate=True)
        self._c = None
        return self

    def workspace_bytes(self, T, cache: KVCache) -> int:
        return lib().fmoe_decoder_workspace_bytes(T, ctypes.byref(self.cstruct()), ctypes.byref(cache.c))

    def forward(self, x: torch.Tensor, cache: KVCache, pos: int, workspace: torch.Tensor, pos_dev=None):
        """In place: x bf16 [T, hidden] (one token per sequence) -> the layer output."""
        T = x.shape[0]
        check(lib().fmoe_decoder_layer_forward(ctypes.byref(self.cstruct()), ctypes.byref(cache.c), _ptr(x), T, pos,
                                               _ptr(pos_dev), _ptr(workspace), workspace.numel(), _stream()))
        return x

    def prefill_workspace_bytes(self, T) -> int:
        return lib().fmoe_decoder_layer_prefill_workspace_bytes(ctypes.byref(self.cstruct()), T)

    def prefill(self, x: torch.Tensor, cache: KVCache, pos0: int, workspace: torch.Tensor, window=None):
        """In place: x bf16 [T, hidden], T prompt tokens of one sequence at
        positions pos0 .. pos0 + T - 1 -> the layer output; the new K/V rows are
        appended to `cache` (batch 1, or a one-sequence view).  window: the
        cache's sliding window by default (None / 0: full causal attention).
        fmoe_decoder_layer_prefill; workspace zero-filled before first use."""
        T = x.shape[0]
        win = cache.window if window is None else window
        prep = prefill_prep(self.experts, x.device)
        check(lib().fmoe_decoder_layer_prefill(ctypes.byref(self.cstruct()), ctypes.byref(cache.c), _ptr(x), T, pos0,
                                               win or 0, _ptr(prep), _ptr(workspace), workspace.numel(), _stream()))
        return x

    def prefill_ep_workspace_bytes(self, T, world: int) -> int:
        return lib().fmoe_decoder_layer_prefill_ep_workspace_bytes(ctypes.byref(self.cstruct()), T, world)

    def prefill_ep(self, comm, x: torch.Tensor, cache: KVCache, pos0: int, workspace: torch.Tensor, window=None):
        """prefill() with this layer's experts being this rank's slice: the routed
        experts run on their owning ranks (fmoe_decoder_layer_prefill_ep; every
        rank calls it with the same T)."""
        T = x.shape[0]
        win = cache.window if window is None else window
        prep = prefill_prep(self.experts, x.device)
        check(lib().fmoe_decoder_layer_prefill_ep(ctypes.byref(self.cstruct()), ctypes.byref(cache.c), comm.handle,
                                                  _ptr(x), T, pos0, win or 0, _ptr(prep), _ptr(workspace),
                                                  workspace.numel(), _stream()))
        return x

    def ep_workspace_bytes(self, T, cache: KVCache, world: int, cap: int) -> int:
        return lib().fmoe_decoder_ep_workspace_bytes(T, ctypes.byref(self.cstruct()), ctypes.byref(cache.c), world,
                                                     cap)

    def forward_ep(self, comm, cap: int, x: torch.Tensor, cache: KVCache, pos: int, workspace: torch.Tensor,
                   pos_dev=None, mode=0, prepared=None):
        """forward() with this layer's experts being this rank's slice: the routed
        experts run on their owning ranks (fmoe_decoder_layer_forward_ep)."""
        T = x.shape[0]
        check(lib().fmoe_decoder_layer_forward_ep(ctypes.byref(self.cstruct()), ctypes.byref(cache.c), comm.handle,
                                                  cap, _ptr(prepared), mode, _ptr(x), T, pos, _ptr(pos_dev),
                                                  _ptr(workspace), workspace.numel(), _stream()))
        return x

    __call__ = forward

    @classmethod
    def random(cls, cfg, full: bool, seed: int, device, experts=None, ep=None):
        """Random-init layer; ep (an EPComm): keep only this rank's expert slice."""
        g = torch.Generator(device=device).manual_seed(seed)
        H = cfg["hidden"]
        D = cfg["full_head_dim"] if full else cfg["sliding_head_dim"]
        Hkv = cfg["full_kv_heads"] if full else cfg["sliding_kv_heads"]
        Hq = cfg["heads"]

        def qlin(out_f, in_f, bits, std=0.02):
            w = torch.randn(out_f, in_f, generator=g, device=device) * std
            return QuantizedLinear.from_float(w, bits)

        def norm(n):
            return (1.0 + 0.1 * torch.randn(n, generator=g, device=device)).to(torch.bfloat16)

        ab, db = cfg["attn_bits"], cfg["dense_bits"]
        q = qlin(Hq * D, H, ab)
        k = qlin(Hkv * D, H, ab)
        v = None if full else qlin(Hkv * D, H, ab)
        o = qlin(H, Hq * D, ab)
        norms = {n: norm(H) for n in ("input", "post_attn", "pre_ff", "post_ff_1", "pre_ff_2", "post_ff_2",
                                      "post_ff")}
        mlp = (qlin(cfg["dense_inter"], H, db), qlin(cfg["dense_inter"], H, db), qlin(H, cfg["dense_inter"], db))
        # O(1) router logits after the root_size scaling: unit-variance router weights
        router = {"proj": qlin(cfg["experts"], H, cfg["router_bits"], std=1.0), "router_scale": norm(H),
                  "per_expert_scale": norm(cfg["experts"]), "root_size": H ** -0.5}
        if experts is None:
            experts = ExpertTable.random(cfg["experts"], H, cfg["expert_inter"], seed=seed + 1, device=device)
            if ep is not None:
                experts = experts.shard(ep.rank, ep.world, copy=True)
        rope_dims = int(D * cfg["full_partial_rotary"]) if full else D
        theta = cfg["full_theta"] if full else cfg["sliding_theta"]
        return cls(q, k, v, o, norm(D), norm(D), norms, mlp, router, experts, Hq, Hkv, D, rope_dims, theta, full,
                   eps=cfg["eps"], layer_scalar=float(0.5 + torch.rand(1, generator=g, device=device).item()),
                   attn_scale=1.0, top_k=cfg["top_k"])


class Gemma4Model:
    """Embedding (6-bit, scaled by sqrt(hidden)), decoder layers with their KV
    caches, final norm and the tied 6-bit lm_head with softcap; greedy decode."""

    def __init__(self, cfg, embed: QuantizedLinear, layers, final_norm, batch, max_positions, kv_mode=KV_BF16,
                 device=None, ep=None, ep_cap=None, ep_mode=2, turbo_bits=0):
        self.cfg = cfg
        self.embed = embed
        self.layers = layers
        self.final_norm = final_norm
        self.batch = batch
        device = torch.device("cuda") if device is None else torch.device(device)
        self.device = device
        self.caches = []
        for i, L in enumerate(layers):
            win = None if getattr(L, "full_attention", L.k_eq_v) else cfg["window"]
            if kv_mode == KV_AFFINE:
                c = KVCache.new_affine(batch, L.num_kv_heads, L.head_dim, max_positions, window=win, device=device)
            else:
                # turbo_bits 2..4: appended rows take the TurboQuant round trip
                # (the reference's default cache, src/main.rs:53, src/cache.rs:290-308)
                c = KVCache(batch, L.num_kv_heads, L.head_dim, max_positions, window=win, turbo_bits=turbo_bits,
                            device=device)
            self.caches.append(c)
        # the lm_head takes at most 8 sequences per call: larger batches run as
        # groups of 8.  A layer call takes up to 64 sequences when every expert is
        # local (its attention half runs per group of 8 inside the library, its
        # feed-forward half once over the batch, so each expert is read once per
        # layer); otherwise (expert-parallel, or FMOE_BATCHED_LAYER=0) groups of 8
        # on views of the same caches
        self.groups = [(b0, min(8, batch - b0)) for b0 in range(0, batch, 8)]
        batched = ep is None and 8 < batch <= 64 and os.environ.get("FMOE_BATCHED_LAYER", "1") != "0"
        self.layer_groups = [(0, batch)] if batched else self.groups
        self.views = [[c.batch_view(b0, nb) for b0, nb in self.groups] if batch > 8 and not batched else [c]
                      for c in self.caches]
        self.ep = ep
        self.ep_cap = min(batch, 8) if ep_cap is None else ep_cap
        # FMOE_EP_P2P (default: peer-memory stores, measured faster than NCCL
        # send / recv at 2 and 4 GPUs) or FMOE_EP_FIXED; both capturable
        self.ep_mode = ep_mode
        if ep is not None and ep_mode == 2:
            ep.ensure_p2p(self.ep_cap, cfg["hidden"], layers[0].top_k)
        if ep is None:
            ws = max(L.workspace_bytes(v.batch, v) for L, vs in zip(layers, self.views) for v in vs)
        else:
            ws = max(L.ep_workspace_bytes(v.batch, v, ep.world, self.ep_cap) for L, vs in zip(layers, self.views)
                     for v in vs)
        if ws == 0:
            raise ValueError("decoder: unsupported layer / cache configuration")
        self.ws = torch.zeros(ws, dtype=torch.uint8, device=device)
        self.lm_ws = torch.zeros(lib().fmoe_lm_head_workspace_bytes(min(batch, 8)) + 256, dtype=torch.uint8,
                                 device=device)
        H, V = cfg["hidden"], embed.out_features
        self.x = torch.zeros(batch, H, dtype=torch.bfloat16, device=device)
        self.logits = torch.empty(batch, V, dtype=torch.float32, device=device)
        self.ids = torch.zeros(batch, dtype=torch.int32, device=device)
        self.pos = 0
        self.pos_dev = torch.zeros(2, dtype=torch.int64, device=device)  # {position, attended slots}
        self._emb_scale = math.sqrt(H)
        self._embed_c = embed.cstruct()
        self._fc = None
        self.sampler = None

    def set_sampler(self, temperature=0.0, top_p=1.0, rep_penalty=1.0, seed=0, window=64):
        """decode_step then draws the next tokens with fmoe_sample (the engine's
        sample(), src/engine.rs:302-355, its last-64-token repetition window
        engine.rs:153-155) instead of the greedy argmax; None-equivalent reset:
        set_sampler(None)."""
        from .sample import Sampler

        if temperature is None:
            self.sampler = None
            return self
        self.sampler = Sampler(self.batch, self.embed.out_features, temperature, top_p, rep_penalty, seed, window,
                               self.device)
        return self

    def tile_weights(self):
        """Tile-layout copies of every decode-GEMV weight (layers and lm_head) for
        the per-row GEMV (fmoe_qlinear).  The decoder's own projections and
        lm_head read the plain layout and do not need them."""
        for L in self.layers:
            L.tile_weights()
        self.embed.tile(accumulate=False)
        self._embed_c = self.embed.cstruct()
        self._fc = None
        return self

    @classmethod
    def random(cls, cfg, batch, max_positions, seed=0, device="cuda", kv_mode=KV_BF16, n_layers=None, ep=None,
               ep_cap=None, ep_mode=2, turbo_bits=0):
        """Random-init model.  ep (an EPComm): every layer keeps only this rank's
        expert slice and decode_step runs the routed experts on their owners."""
        n_layers = cfg["layers"] if n_layers is None else n_layers
        layers = [Gemma4DecoderLayer.random(cfg, layer_is_full(cfg, i), seed + 100 * i, device, ep=ep)
                  for i in range(n_layers)]
        g = torch.Generator(device=device).manual_seed(seed + 7)
        rows = []
        # the [vocab, hidden] embedding in row blocks (bounded fp32 scratch)
        V, H = cfg["vocab"], cfg["hidden"]
        blk = 32768
        wq = torch.empty(V, H * cfg["embed_bits"] // 32, dtype=torch.int32, device=device)
        sc = torch.empty(V, H // 64, dtype=torch.bfloat16, device=device)
        bi = torch.empty_like(sc)
        from . import quantize
        for r0 in range(0, V, blk):
            w = torch.randn(min(blk, V - r0), H, generator=g, device=device) * 0.02
            a, b_, c_ = quantize(w, cfg["embed_bits"])
            wq[r0:r0 + w.shape[0]] = a
            sc[r0:r0 + w.shape[0]] = b_
            bi[r0:r0 + w.shape[0]] = c_
            rows.append(None)
        embed = QuantizedLinear(wq, sc, bi, cfg["embed_bits"], 64, in_features=H)
        final_norm = (1.0 + 0.1 * torch.randn(H, generator=g, device=device)).to(torch.bfloat16)
        return cls(cfg, embed, layers, final_norm, batch, max_positions, kv_mode, device, ep, ep_cap, ep_mode,
                   turbo_bits)

    def _fused(self):
        if self._fc is None:
            if self.ep is not None:
                raise ValueError("decode_step_fused: all experts must be local")
            if self.batch != 1:
                raise ValueError("decode_step_fused: batch 1 only")
            n = len(self.layers)
            lay = (DecoderLayerC * n)(*[L.cstruct() for L in self.layers])
            cac = (KvCacheC * n)(*[c.c for c in self.caches])
            mc = DecodeModelC(n, 0, lay, cac, self._embed_c, _ptr(self.final_norm), self.cfg["eps"],
                              self.cfg["softcap"], self._emb_scale)
            nbytes = lib().fmoe_decode_step_workspace_bytes(ctypes.byref(mc))
            if nbytes == 0:
                check(lib().fmoe_decode_step_prepare(ctypes.byref(mc), None, 0))
            ws = torch.zeros(nbytes, dtype=torch.uint8, device=self.device)
            check(lib().fmoe_decode_step_prepare(ctypes.byref(mc), _ptr(ws), nbytes))
            self._fc = (mc, lay, cac, ws)
        return self._fc

    def decode_step_fused(self):
        """One greedy decode step (batch 1) as a single persistent kernel:
        ids -> next ids (in self.ids); the position advances on the device
        (pos_dev) and on the host."""
        mc, _, _, ws = self._fused()
        check(lib().fmoe_decode_step(ctypes.byref(mc), _ptr(self.ids), _ptr(self.logits), _ptr(self.pos_dev), _ptr(ws),
                                     ws.numel(), _stream()))
        self.pos += 1
        for cache in self.caches:
            cache._offset = self.pos
        return self.ids

    def status(self, clear: bool = False) -> int:
        """Status word of the layered step's workspace (0: ok; a bounded device
        wait that gave up — e.g. a peer-memory exchange flag that never came —
        leaves FMOE_ERR_TIMEOUT; synchronises)."""
        return lib().fmoe_workspace_status(_ptr(self.ws), int(clear), _stream())

    def fused_status(self, clear: bool = False) -> int:
        """Status word of the fused step's workspace (0: ok; synchronises)."""
        return lib().fmoe_workspace_status(_ptr(self._fused()[3]), int(clear), _stream())

    def prefill(self, tokens: torch.Tensor, chunk: int = 2048):
        """Run the prompt of every sequence through the model (one sequence at a
        time, in chunks of at most `chunk` tokens through all layers), appending
        its K/V rows, and leave each sequence's next greedy token in self.ids.
        Expert-parallel models: collective, every rank with prompts of the same
        length (the routed experts run on their owning ranks).
        tokens: int32 [batch, T] (or [T] for batch 1), all sequences the same
        length, starting at the current position.  TextModel::forward with
        l = T (src/model/mod.rs:135-254) followed by Model::forward's lm_head on
        the last position (mod.rs:336-362)."""
        tok = tokens.to(device=self.device, dtype=torch.int32)
        if tok.dim() == 1:
            tok = tok.view(1, -1)
        B, T = tok.shape
        if B != self.batch or T < 1:
            raise ValueError(f"prefill: tokens {tuple(tok.shape)} for batch {self.batch}")
        chunk = max(1, min(chunk, T))
        if self.ep is None:
            need = max(L.prefill_workspace_bytes(chunk) for L in self.layers)
        else:  # every rank runs the same chunks (the expert exchange is collective)
            need = max(L.prefill_ep_workspace_bytes(chunk, self.ep.world) for L in self.layers)
        if need == 0:
            raise ValueError("prefill: unsupported layer configuration")
        if getattr(self, "_pf_ws", None) is None or self._pf_ws.numel() < need:
            self._pf_ws = torch.zeros(need, dtype=torch.uint8, device=self.device)
        H = self.cfg["hidden"]
        c = self._embed_c
        pos0 = self.pos
        for b in range(B):
            views = [cache.batch_view(b, 1) if cache.batch > 1 else cache for cache in self.caches]
            x = None
            for s0 in range(0, T, chunk):
                n = min(chunk, T - s0)
                x = torch.empty(n, H, dtype=torch.bfloat16, device=self.device)
                ids = tok[b, s0:s0 + n].contiguous()
                check(lib().fmoe_embed_rows(ctypes.byref(c), _ptr(ids), n, self._emb_scale, _ptr(x), _stream()))
                for L, v in zip(self.layers, views):
                    if self.ep is None:
                        L.prefill(x, v, pos0 + s0, self._pf_ws)
                    else:
                        L.prefill_ep(self.ep, x, v, pos0 + s0, self._pf_ws)
            check(lib().fmoe_lm_head(ctypes.byref(c), _ptr(self.final_norm), self.cfg["eps"], _ptr(x[-1:]), 1,
                                     self.cfg["softcap"], _ptr(self.logits[b:b + 1]), _ptr(self.ids[b:b + 1]), None,
                                     _ptr(self.lm_ws), self.lm_ws.numel(), _stream()))
        self.set_position(pos0 + T)
        for cache in self.caches:
            cache._offset = self.pos
        return self.ids

    def set_sparse_v_threshold(self, tau: float):
        """Model::set_sparse_v_threshold (src/model/mod.rs:367-372): every
        layer's decode attention zeroes the softmax weights below tau (no
        renormalisation); 0 turns it off; prefill is unaffected.  Applies to the
        layered decode path (bf16 / TurboQuant caches); re-capture any CUDA graph
        of decode_step afterwards."""
        if not tau >= 0.0:
            raise ValueError(f"sparse-V threshold {tau}")
        for L in self.layers:
            L.sparse_v_tau = float(tau)
            L._c = None
        self._fc = None

    def set_position(self, pos: int):
        self.pos = pos
        n = min(pos + 1, 1 << 62)
        self.pos_dev.copy_(torch.tensor([pos, n], dtype=torch.int64))

    def decode_step(self, device_pos=False):
        """One greedy decode step for every sequence: ids -> next ids (in self.ids).
        device_pos=True reads / advances the position on the device (graph replay)."""
        c = self._embed_c
        check(lib().fmoe_embed_rows(ctypes.byref(c), _ptr(self.ids), self.batch, self._emb_scale, _ptr(self.x),
                                    _stream()))
        pd = self.pos_dev if device_pos else None
        for L, views in zip(self.layers, self.views):
            for (b0, nb), v in zip(self.layer_groups, views):
                x = self.x[b0:b0 + nb]
                if self.ep is None:
                    L.forward(x, v, self.pos, self.ws, pd)
                else:
                    L.forward_ep(self.ep, self.ep_cap, x, v, self.pos, self.ws, pd, mode=self.ep_mode)
        for i, (b0, nb) in enumerate(self.groups):  # the last call advances the device position
            check(lib().fmoe_lm_head(ctypes.byref(c), _ptr(self.final_norm), self.cfg["eps"], _ptr(self.x[b0:b0 + nb]),
                                     nb, self.cfg["softcap"], _ptr(self.logits[b0:b0 + nb]), _ptr(self.ids[b0:b0 + nb]),
                                     _ptr(pd if i == len(self.groups) - 1 else None), _ptr(self.lm_ws),
                                     self.lm_ws.numel(), _stream()))
        if self.sampler is not None:  # the draw replaces the lm_head's greedy ids
            self.sampler(self.logits, out=self.ids)
        if not device_pos:
            self.pos += 1
            for cache in self.caches:
                cache._offset = self.pos
        return self.ids
