"""CPU oracle for libfmoe — TEST INFRASTRUCTURE ONLY.

numpy/ctypes front end of fmoe_oracle.cpp, a C++ restatement of the arithmetic
flash-moe's MoE / KV-cache path performs through MLX (each C function cites the
reference call site it follows).  Only tests/, __graft_entry__.smoke() and
bench.py's CPU-baseline leg may use it, and only as the checker.

PARITY UNPINNED: the reference ships no tests, golden vectors or fixtures, and
its arithmetic lives in MLX (mlx-rs 0.25.3 / mlx-sys 0.2.0), which cannot run
here; see fmoe_oracle.cpp's header for the numeric definitions fixed instead.
bf16 arrays are carried as numpy uint16 bit patterns.
"""
from __future__ import annotations

import ctypes
import os

import numpy as np

from . import build as _build

_lib = None


def lib():
    global _lib
    if _lib is None:
        path = _build.OUT
        if not os.path.exists(path):
            _build.build()
        _lib = ctypes.CDLL(path)
    return _lib


def _p(a):
    return None if a is None else a.ctypes.data_as(ctypes.c_void_p)


def num_threads() -> int:
    return lib().orc_num_threads()


def set_num_threads(n: int) -> None:
    lib().orc_set_num_threads(ctypes.c_int(n))


def f32_to_bf16(x) -> np.ndarray:
    x = np.ascontiguousarray(x, dtype=np.float32)
    y = np.empty(x.shape, np.uint16)
    lib().orc_f32_to_bf16(_p(x), ctypes.c_int64(x.size), _p(y))
    return y


def bf16_to_f32(x) -> np.ndarray:
    x = np.ascontiguousarray(x, dtype=np.uint16)
    y = np.empty(x.shape, np.float32)
    lib().orc_bf16_to_f32(_p(x), ctypes.c_int64(x.size), _p(y))
    return y


def quantize(w: np.ndarray, bits: int, group: int = 64):
    """MLX-affine quantisation of fp32 [rows, cols] -> (wq uint32, scales bf16, biases bf16)."""
    w = np.ascontiguousarray(w, dtype=np.float32)
    rows, cols = w.shape
    wq = np.zeros((rows, cols * bits // 32), np.uint32)
    s = np.empty((rows, cols // group), np.uint16)
    b = np.empty_like(s)
    lib().orc_quantize(_p(w), ctypes.c_int64(rows), ctypes.c_int64(cols), bits, group, _p(wq), _p(s), _p(b))
    return wq, s, b


def dequantize(wq, s, b, cols: int, bits: int, group: int = 64) -> np.ndarray:
    wq = np.ascontiguousarray(wq, dtype=np.uint32)
    rows = wq.shape[0]
    out = np.empty((rows, cols), np.uint16)
    lib().orc_dequantize(_p(wq), _p(np.ascontiguousarray(s)), _p(np.ascontiguousarray(b)), ctypes.c_int64(rows),
                         ctypes.c_int64(cols), bits, group, _p(out))
    return out


def qmatmul(x_bf16, wq, s, b, in_features: int, bits: int, group: int = 64) -> np.ndarray:
    """fp32 [T, out] = x . W^T (exact per-group form, double accumulation)."""
    x = np.ascontiguousarray(x_bf16, dtype=np.uint16)
    T = x.shape[0]
    out = wq.shape[0]
    y = np.empty((T, out), np.float32)
    lib().orc_qmatmul(_p(x), ctypes.c_int64(T), _p(np.ascontiguousarray(wq, np.uint32)), _p(np.ascontiguousarray(s)),
                      _p(np.ascontiguousarray(b)), ctypes.c_int64(out), ctypes.c_int64(in_features), bits, group, _p(y))
    return y


def matmul_bf16(x_bf16, w_bf16) -> np.ndarray:
    x = np.ascontiguousarray(x_bf16, np.uint16)
    w = np.ascontiguousarray(w_bf16, np.uint16)
    y = np.empty((x.shape[0], w.shape[0]), np.float32)
    lib().orc_matmul_bf16(_p(x), ctypes.c_int64(x.shape[0]), _p(w), ctypes.c_int64(w.shape[0]),
                          ctypes.c_int64(w.shape[1]), _p(y))
    return y


def router(x_bf16, wr, k: int, wr_bits: int = 16, wr_s=None, wr_b=None, group=64, logit_bias=None, use_norm=False,
           root_size=0.0, eps=1e-6, router_scale=None, per_expert_scale=None):
    """Gemma4MoeBlock router (src/model/moe.rs:324-345) -> (ids, weights, logits)."""
    x = np.ascontiguousarray(x_bf16, np.uint16)
    T, H = x.shape
    E = wr.shape[0]
    ids = np.empty((T, k), np.int32)
    w = np.empty((T, k), np.float32)
    lg = np.empty((T, E), np.float32)
    lib().orc_router(_p(x), T, H, E, _p(np.ascontiguousarray(wr)), _p(wr_s), _p(wr_b), wr_bits, group,
                     _p(None if logit_bias is None else np.ascontiguousarray(logit_bias, np.float32)), int(use_norm),
                     ctypes.c_float(root_size), ctypes.c_float(eps),
                     _p(None if router_scale is None else np.ascontiguousarray(router_scale, np.uint16)),
                     _p(None if per_expert_scale is None else np.ascontiguousarray(per_expert_scale, np.uint16)), k,
                     _p(ids), _p(w), _p(lg))
    return ids, w, lg


def moe_experts(x_bf16, ids, weights, expert_buf: np.ndarray, stride: int, offsets, hidden: int, inter: int, bits=4,
                group=64, want_act=False):
    """Routed experts + combine (src/model/moe.rs:424-466) -> (y fp32, y bf16[, act bf16 [T,k,I]])."""
    x = np.ascontiguousarray(x_bf16, np.uint16)
    T = x.shape[0]
    k = ids.shape[1]
    y32 = np.empty((T, hidden), np.float32)
    y16 = np.empty((T, hidden), np.uint16)
    act = np.empty((T, k, inter), np.uint16) if want_act else None
    offs = (ctypes.c_int64 * 9)(*offsets)
    lib().orc_moe_experts(_p(x), T, hidden, inter, k, _p(np.ascontiguousarray(ids, np.int32)),
                          _p(np.ascontiguousarray(weights, np.float32)), _p(np.ascontiguousarray(expert_buf, np.uint8)),
                          ctypes.c_int64(stride), offs, bits, group, _p(y32), _p(y16), _p(act))
    return (y32, y16, act) if want_act else (y32, y16)


def hadamard(n: int) -> np.ndarray:
    h = np.empty((n, n), np.float32)
    lib().orc_hadamard(n, _p(h))
    return h


def signs(n: int, seed: int = 42) -> np.ndarray:
    s = np.empty(n, np.float32)
    lib().orc_signs(n, ctypes.c_uint64(seed), _p(s))
    return s


def lloyd_max(bits: int):
    c = np.empty(16, np.float32)
    b = np.empty(15, np.float32)
    n = lib().orc_lloyd_max(bits, _p(c), _p(b))
    return c[:n].copy(), b[:n - 1].copy()


def turbo_round_trip(v_bf16, bits: int):
    """TurboQuant round trip (src/cache.rs:94-129) of rows [..., D] -> (out bf16, idx uint8, norms f32)."""
    v = np.ascontiguousarray(v_bf16, np.uint16)
    D = v.shape[-1]
    rows = v.size // D
    out = np.empty(v.shape, np.uint16)
    idx = np.empty(v.shape, np.uint8)
    nrm = np.empty(v.shape[:-1], np.float32)
    lib().orc_turbo_round_trip(_p(v), ctypes.c_int64(rows), D, bits, _p(out), _p(idx), _p(nrm))
    return out, idx, nrm


def wht_rows(x_f32) -> np.ndarray:
    x = np.ascontiguousarray(x_f32, np.float32)
    D = x.shape[-1]
    out = np.empty_like(x)
    lib().orc_wht_rows(_p(x), ctypes.c_int64(x.size // D), D, _p(out))
    return out


def kv_quant_affine(v_bf16, bits: int, group: int = 64):
    """WHT-rotate then MLX-affine quantise rows [..., D] -> (wq, scales, biases)."""
    v = np.ascontiguousarray(v_bf16, np.uint16)
    D = v.shape[-1]
    rows = v.size // D
    wq = np.zeros((rows, D * bits // 32), np.uint32)
    s = np.empty((rows, D // group), np.uint16)
    b = np.empty_like(s)
    lib().orc_kv_quant_affine(_p(v), ctypes.c_int64(rows), D, bits, group, _p(wq), _p(s), _p(b))
    return wq, s, b


def attn_decode_affine(q_bf16, Hkv, Tcap, t_lo, t_hi, kq, ks, kb, kbits, vq, vs, vb, vbits, scale, group=64):
    q = np.ascontiguousarray(q_bf16, np.uint16)
    B, Hq, D = q.shape
    out = np.empty((B, Hq, D), np.float32)
    lib().orc_attn_decode_affine(_p(q), B, Hq, Hkv, D, ctypes.c_int64(Tcap), _p(np.ascontiguousarray(t_lo, np.int32)),
                                 _p(np.ascontiguousarray(t_hi, np.int32)), _p(kq), _p(ks), _p(kb), kbits, _p(vq), _p(vs),
                                 _p(vb), vbits, group, ctypes.c_float(scale), _p(out))
    return out


def attn_decode_bf16(q_bf16, Hkv, Tcap, t_lo, t_hi, k_bf16, v_bf16, scale, tau=0.0):
    q = np.ascontiguousarray(q_bf16, np.uint16)
    B, Hq, D = q.shape
    out = np.empty((B, Hq, D), np.float32)
    lib().orc_attn_decode_bf16(_p(q), B, Hq, Hkv, D, ctypes.c_int64(Tcap), _p(np.ascontiguousarray(t_lo, np.int32)),
                               _p(np.ascontiguousarray(t_hi, np.int32)), _p(np.ascontiguousarray(k_bf16, np.uint16)),
                               _p(np.ascontiguousarray(v_bf16, np.uint16)), ctypes.c_float(scale), ctypes.c_float(tau),
                               _p(out))
    return out


# ---------------------------------------------------------------------------
# Decoder layer (config: Gemma-4 decode step), composed from the C pieces.


def rms_norm(x_bf16, w_bf16=None, eps=1e-6):
    """fast::rms_norm / RMSNormNoScale (src/model/norm.rs:11-29) over the last axis."""
    x = np.ascontiguousarray(x_bf16, np.uint16)
    n = x.shape[-1]
    y = np.empty_like(x)
    w = None if w_bf16 is None else np.ascontiguousarray(w_bf16, np.uint16)
    lib().orc_rms_norm(_p(x), ctypes.c_int64(x.size // n), n, _p(w), ctypes.c_float(eps), _p(y))
    return y


def rope(x_bf16, dims, theta, pos):
    """fast::rope (traditional=false), src/model/gemma4_attention.rs:74-81, over the last axis."""
    x = np.ascontiguousarray(x_bf16, np.uint16)
    D = x.shape[-1]
    y = np.empty_like(x)
    lib().orc_rope(_p(x), ctypes.c_int64(x.size // D), D, dims, ctypes.c_double(theta), ctypes.c_int64(pos), _p(y))
    return y


def _bf(x_f32):
    return f32_to_bf16(np.asarray(x_f32, np.float32))


def _f(x_bf16):
    return bf16_to_f32(x_bf16)


def _gelu(g):
    g = g.astype(np.float64)
    return 0.5 * g * (1.0 + np.tanh(0.7978845608028654 * (g + 0.044715 * g ** 3)))


def _qlin(x_bf16, w):
    """w = (wq uint32, scales, biases, in_features, bits) -> bf16 output (MLX qmm output dtype)."""
    wq, s, b, in_f, bits = w
    return _bf(qmatmul(x_bf16, wq, s, b, in_f, bits))


def decoder_layer(x, L, cache_k, cache_v, pos, cfg):
    """One decode step of DecoderLayer::forward_gemma4 (src/model/mod.rs:67-119) for
    T sequences (one token each).

    x: bf16 [T, H]; L: dict of weights (q/k/v/o/gate/up/down as _qlin tuples,
    bf16 norms, router (wr, bits, scale, pes, root), experts (buf, stride, offsets));
    cache_k / cache_v: bf16 [T, Hkv, cap, D], updated at slot pos % cap — or,
    with cfg["kv_mode"] == "affine", the tuples (codes, scales, biases) of the
    WHT-rotated 4-bit K / 8-bit V cache ([T, Hkv, cap, ...] each), the new row
    quantised by kv_quant_affine (src/cache.rs:266-310 with the affine store).
    cfg["turbo_bits"] (bf16 caches only): the new K / V rows pass through the
    TurboQuant round trip before they are stored (src/cache.rs:290-308).
    cfg: heads, kv_heads, head_dim, rope_dims, rope_theta, eps, k_eq_v, scalar,
    attn_scale, top_k, hidden, inter_expert.  Returns (x_out bf16, q_rot bf16).
    """
    T, H = x.shape
    Hq, Hkv, D, eps = cfg["heads"], cfg["kv_heads"], cfg["head_dim"], cfg["eps"]
    # attention block (gemma4_attention.rs:46-112)
    xn = rms_norm(x, L["input_norm"], eps)
    q = _qlin(xn, L["q"]).reshape(T, Hq, D)
    k = _qlin(xn, L["k"]).reshape(T, Hkv, D)
    v = k.copy() if cfg["k_eq_v"] else _qlin(xn, L["v"]).reshape(T, Hkv, D)
    q = rope(rms_norm(q, L["q_norm"], eps), cfg["rope_dims"], cfg["rope_theta"], pos)
    k = rope(rms_norm(k, L["k_norm"], eps), cfg["rope_dims"], cfg["rope_theta"], pos)
    v = rms_norm(v, None, eps)
    lo = np.zeros(T, np.int32)
    if cfg.get("kv_mode", "bf16") == "affine":
        cap = cache_k[0].shape[2]
        for arr, new in zip(cache_k + cache_v, kv_quant_affine(k, 4) + kv_quant_affine(v, 8)):
            arr[:, :, pos % cap] = new.reshape(arr[:, :, pos % cap].shape)
        hi = np.full(T, min(pos + 1, cap), np.int32)
        att = attn_decode_affine(q, Hkv, cap, lo, hi, *cache_k, 4, *cache_v, 8, cfg["attn_scale"])
    else:
        tb = cfg.get("turbo_bits", 0)
        if tb:
            k = turbo_round_trip(k, tb)[0]
            v = turbo_round_trip(v, tb)[0]
        cap = cache_k.shape[2]
        cache_k[:, :, pos % cap] = k
        cache_v[:, :, pos % cap] = v
        hi = np.full(T, min(pos + 1, cap), np.int32)
        # cfg["sparse_v_tau"] > 0: the decode-only gate of gemma4_attention.rs:91-93, 196-234
        att = attn_decode_bf16(q, Hkv, cap, lo, hi, cache_k, cache_v, cfg["attn_scale"], tau=cfg.get("sparse_v_tau", 0.0))
    return _ff_block(x, _bf(att).reshape(T, Hq * D), L, cfg), q


def _ff_block(x, att, L, cfg):
    """o_proj, residual and the feed-forward block of forward_gemma4 (mod.rs:80-118)
    for T rows: x bf16 [T, H] the layer input, att bf16 [T, Hq * D]."""
    T, H = x.shape
    eps = cfg["eps"]
    o = _qlin(att, L["o"])
    h = _bf(_f(x) + _f(rms_norm(o, L["post_attn_norm"], eps)))
    # feed-forward block: dense MLP + MoE in parallel (mod.rs:92-118)
    h1 = rms_norm(h, L["pre_ff_norm"], eps)
    h2 = rms_norm(h, L["pre_ff_norm_2"], eps)
    g = _qlin(h1, L["gate"])
    u = _qlin(h1, L["up"])
    act = _bf(_gelu(_f(g)) * _f(u))
    d = _qlin(act, L["down"])
    wr, wr_bits, rscale, pes, root = L["router"]
    ids, wts, logits = router(h2, wr, cfg["top_k"], wr_bits, use_norm=True, root_size=root, eps=eps,
                              router_scale=rscale, per_expert_scale=pes, logit_bias=L.get("logit_bias"))
    cfg["_router_logits"] = logits
    buf, stride, offs = L["experts"]
    y, _ = moe_experts(h2, ids, wts, buf, stride, offs, H, cfg["inter_expert"])
    moe = _bf(y)
    s = _bf(_f(rms_norm(d, L["post_ff_norm_1"], eps)) + _f(rms_norm(moe, L["post_ff_norm_2"], eps)))
    out = _bf(_f(h) + _f(rms_norm(s, L["post_ff_norm"], eps)))
    sc = _f(_bf(np.float32([cfg["scalar"]])))[0]
    return _bf(_f(out) * sc)


def mlp(x_bf16, gate, up, down):
    """GeLUMLP::forward (src/model/mlp.rs:28-41): down(gelu_tanh(gate(x)) * up(x)), bf16 [T, H]."""
    act = _bf(_gelu(_f(_qlin(x_bf16, gate))) * _f(_qlin(x_bf16, up)))
    return _qlin(act, down)


def attn_prefill_bf16(q_bf16, k_ring, v_ring, k_new, v_new, pos0: int, window: int, scale: float) -> np.ndarray:
    """SDPA of T new tokens of one sequence over the stored rows plus the new
    ones, as the reference's prefill runs it: update_and_fetch returns
    concat(stored, new) (src/cache.rs:266-288) and the additive mask of
    create_attention_mask / create_sliding_mask (src/model/mod.rs:682-753)
    admits key position j for the query at position p iff j <= p and, with a
    window, p - j < window; scaled_dot_product_attention then takes a softmax
    over the admitted keys (gemma4_attention.rs:95-104).  float64 throughout.

    q bf16 [T, Hq, D]; k_ring / v_ring bf16 [Hkv, cap, D] (position j < pos0 at
    slot j % cap); k_new / v_new bf16 [Hkv, T, D].  Returns f32 [T, Hq, D]."""
    return _attn_prefill(_f(q_bf16), _f(k_ring), _f(v_ring), _f(k_new), _f(v_new), pos0, window, scale)


def attn_prefill_affine(q_bf16, k_ring, v_ring, k_new, v_new, pos0: int, window: int, scale: float):
    """attn_prefill_bf16 over the WHT-rotated affine K4 / V8 cache: the stored
    rows are dequantised (rotated basis), the new rows take the cache's own
    round trip (rotate, quantise as kv_quant_affine, dequantise), the query is
    rotated the same way and the output rotated back (the normalised WHT is its
    own inverse), as the decode attention over this cache does.

    k_ring / v_ring: (codes, scales, biases) [Hkv, cap, ...]; k_new / v_new bf16
    [Hkv, T, D].  Returns (out f32 [T, Hq, D], new K codes, new V codes), the
    codes as (wq, s, b) [Hkv, T, ...] for the cache's slots."""
    q = np.ascontiguousarray(q_bf16, np.uint16)
    T, Hq, D = q.shape
    Hkv, cap = k_ring[0].shape[0], k_ring[0].shape[1]

    def deq(arrs, bits, rows):
        wq, sc, bi = (a.reshape(rows, -1) for a in arrs)
        return _f(dequantize(wq, sc, bi, D, bits))

    kc = tuple(a.reshape(Hkv, T, -1) for a in kv_quant_affine(k_new, 4))
    vc = tuple(a.reshape(Hkv, T, -1) for a in kv_quant_affine(v_new, 8))
    kr = deq(k_ring, 4, Hkv * cap).reshape(Hkv, cap, D)
    vr = deq(v_ring, 8, Hkv * cap).reshape(Hkv, cap, D)
    kn = deq(kc, 4, Hkv * T).reshape(Hkv, T, D)
    vn = deq(vc, 8, Hkv * T).reshape(Hkv, T, D)
    qr = wht_rows(_f(q).reshape(T * Hq, D)).reshape(T, Hq, D)
    out = _attn_prefill(qr, kr, vr, kn, vn, pos0, window, scale)
    return wht_rows(out.reshape(T * Hq, D)).reshape(T, Hq, D), kc, vc


def _attn_prefill(q, kr, vr, kn, vn, pos0, window, scale):
    """The masked softmax attention of attn_prefill_bf16 on float arrays."""
    q = np.asarray(q, np.float64)
    T, Hq, D = q.shape
    Hkv, cap = kr.shape[0], kr.shape[1]
    R = Hq // Hkv
    lo = max(0, pos0 - window + 1) if window else 0
    old = np.arange(lo, pos0, dtype=np.int64)
    K = np.concatenate([kr[:, old % cap], kn], axis=1).astype(np.float64)
    V = np.concatenate([vr[:, old % cap], vn], axis=1).astype(np.float64)
    kpos = np.concatenate([old, pos0 + np.arange(T, dtype=np.int64)])
    qpos = pos0 + np.arange(T, dtype=np.int64)
    ok = kpos[None, :] <= qpos[:, None]
    if window:
        ok &= (qpos[:, None] - kpos[None, :]) < window
    out = np.empty((T, Hq, D), np.float64)
    for h in range(Hq):
        s = (q[:, h] @ K[h // R].T) * scale
        s = np.where(ok, s, -np.inf)
        s -= s.max(axis=1, keepdims=True)
        p = np.exp(s)
        p /= p.sum(axis=1, keepdims=True)
        out[:, h] = p @ V[h // R]
    return out.astype(np.float32)


def decoder_layer_prefill(x, L, cache_k, cache_v, pos0: int, window: int, cfg, new_rows=None):
    """Prefill of T prompt tokens of one sequence through DecoderLayer::
    forward_gemma4 (src/model/mod.rs:67-119) at positions pos0 .. pos0 + T - 1.

    x bf16 [T, H]; L, cfg as decoder_layer (cfg["turbo_bits"] puts the new K / V
    rows through the TurboQuant round trip, src/cache.rs:290-308);
    cache_k / cache_v bf16 [1, Hkv, cap, D], updated with the new rows at slots
    (pos0 + t) % cap — or, with cfg["kv_mode"] == "affine", the (codes, scales,
    biases) tuples of the rotated K4 / V8 cache, attended by attn_prefill_affine
    and updated with the new rows' codes.  window 0: full causal attention.  The new rows computed here
    are left in cfg["_new_rows"] ([Hkv, T, D] each); new_rows = (k, v) replaces them
    in attention and in the cache (a checker comparing the rows on their own can
    then hold the rest of the layer to the rows actually stored).  Returns
    (x_out bf16, q_rot bf16)."""
    T, H = x.shape
    Hq, Hkv, D, eps = cfg["heads"], cfg["kv_heads"], cfg["head_dim"], cfg["eps"]
    xn = rms_norm(x, L["input_norm"], eps)
    q = _qlin(xn, L["q"]).reshape(T, Hq, D)
    k = _qlin(xn, L["k"]).reshape(T, Hkv, D)
    v = k.copy() if cfg["k_eq_v"] else _qlin(xn, L["v"]).reshape(T, Hkv, D)
    qn = rms_norm(q, L["q_norm"], eps)
    kn = rms_norm(k, L["k_norm"], eps)
    q = np.stack([rope(qn[t], cfg["rope_dims"], cfg["rope_theta"], pos0 + t) for t in range(T)])
    k = np.stack([rope(kn[t], cfg["rope_dims"], cfg["rope_theta"], pos0 + t) for t in range(T)])
    v = rms_norm(v, None, eps)
    cfg["_pre_round_trip"] = (k.copy(), v.copy())  # [T, Hkv, D]
    tb = cfg.get("turbo_bits", 0)
    if tb:
        k = turbo_round_trip(k, tb)[0]
        v = turbo_round_trip(v, tb)[0]
    k_new, v_new = np.ascontiguousarray(k.transpose(1, 0, 2)), np.ascontiguousarray(v.transpose(1, 0, 2))
    cfg["_new_rows"] = (k_new, v_new)
    if new_rows is not None:
        k_new, v_new = (np.ascontiguousarray(r, np.uint16) for r in new_rows)
    if cfg.get("kv_mode", "bf16") == "affine":
        att, kc, vc = attn_prefill_affine(q, tuple(a[0] for a in cache_k), tuple(a[0] for a in cache_v), k_new,
                                          v_new, pos0, window, cfg["attn_scale"])
        cap = cache_k[0].shape[2]
        for t in range(max(0, T - cap), T):
            for arr, new in zip(cache_k + cache_v, kc + vc):
                arr[0, :, (pos0 + t) % cap] = new[:, t]
        return _ff_block(x, _bf(att).reshape(T, Hq * D), L, cfg), q
    att = attn_prefill_bf16(q, cache_k[0], cache_v[0], k_new, v_new, pos0, window, cfg["attn_scale"])
    cap = cache_k.shape[2]
    for t in range(max(0, T - cap), T):
        cache_k[0, :, (pos0 + t) % cap] = k_new[:, t]
        cache_v[0, :, (pos0 + t) % cap] = v_new[:, t]
    return _ff_block(x, _bf(att).reshape(T, Hq * D), L, cfg), q


def lm_head(x, embed, final_norm, eps, softcap):
    """Final norm + tied lm_head + softcap (mod.rs:254, 336-362) -> (logits f32, argmax ids)."""
    xn = rms_norm(x, final_norm, eps)
    wq, s, b, in_f, bits = embed
    lg = _f(_bf(qmatmul(xn, wq, s, b, in_f, bits)))
    if softcap > 0:
        lg = _f(_bf(_f(_bf(np.tanh(_f(_bf(lg / np.float32(softcap))).astype(np.float64)))) * np.float32(softcap)))
    return lg, np.argmax(lg, axis=1).astype(np.int32)
