"""GPU parity: sparse-V decode attention (fmoe_attn_decode_sparse_v) against the
oracle's gated softmax (orc_attn_decode_bf16 with tau), the reference's
sparse_v_attention (src/model/gemma4_attention.rs:196-234): weights below tau
are zeroed and the rest are not renormalised.

Tolerance: max |gpu - oracle| / max |oracle| <= 1e-2 (bf16 output, fp32
against float64 softmax).  Each tau is placed in the middle of the gap between
the two softmax weights (computed here in float64) nearest to the requested
value, so no weight sits close enough to tau for the fp32 / float64
difference to flip the gate.
"""
import numpy as np
import pytest
import torch

from gpu_util import max_rel_err, to_np_bf16

pytestmark = pytest.mark.gpu


def _probs(orc, q, k, v, n, Hkv, scale):
    """Softmax weights [B, Hq, n] in float64, as the oracle forms them."""
    qf = orc.bf16_to_f32(q).astype(np.float64)
    kf = orc.bf16_to_f32(k[:, :, :n]).astype(np.float64)
    B, Hq, D = qf.shape
    R = Hq // Hkv
    s = np.einsum("bhd,bhtd->bht", qf, np.repeat(kf, R, axis=1)) * scale
    s -= s.max(axis=2, keepdims=True)
    p = np.exp(s)
    return p / p.sum(axis=2, keepdims=True)


def _robust_tau(p, target):
    """The midpoint of the gap between the weights just below and above target."""
    flat = np.sort(p.ravel())
    i = int(np.searchsorted(flat, target))
    lo, hi = flat[max(i - 1, 0)], flat[min(i, flat.size - 1)]
    return float(0.5 * (lo + hi)), float(hi - lo)


@pytest.mark.parametrize("B,Hkv,Hq,D,cap,n,taus", [
    (2, 8, 16, 256, 1024, 700, (0.002, 0.01)),
    (1, 2, 16, 512, 2048, 1500, (0.001, 0.005)),
])
def test_sparse_v_matches_oracle(fm, orc, dev, B, Hkv, Hq, D, cap, n, taus):
    g = torch.Generator(device=dev).manual_seed(D + n)
    cache = fm.KVCache(B, Hkv, D, cap, device=dev)
    cache.update(torch.randn(B, Hkv, n, D, generator=g, device=dev).to(torch.bfloat16),
                 torch.randn(B, Hkv, n, D, generator=g, device=dev).to(torch.bfloat16))
    q = (torch.randn(B, Hq, D, generator=g, device=dev) * 0.15).to(torch.bfloat16)
    a = cache.arrays()
    k, v, qn = to_np_bf16(a["k"]), to_np_bf16(a["v"]), to_np_bf16(q)
    p = _probs(orc, qn, k, v, n, Hkv, 1.0)
    lo, hi = np.zeros(B, np.int32), np.full(B, n, np.int32)
    dense = cache.attend(q, 1.0, n_valid=n)
    got0 = cache.attend_sparse_v(q, 0.0, n_valid=n)
    torch.cuda.synchronize()
    assert max_rel_err(orc.bf16_to_f32(to_np_bf16(got0)), orc.bf16_to_f32(to_np_bf16(dense))) <= 1e-2
    for target in taus:
        tau, gap = _robust_tau(p, target)
        kept = float((p >= tau).mean())
        got = cache.attend_sparse_v(q, tau, n_valid=n)
        torch.cuda.synchronize()
        want = orc.attn_decode_bf16(qn, Hkv, cap, lo, hi, k, v, 1.0, tau=tau)
        err = max_rel_err(orc.bf16_to_f32(to_np_bf16(got)), want)
        print(f"tau {tau:.5f} (gap {gap:.2e}): {kept:.3f} of the weights kept, max rel err {err:.2e}")
        assert 0.0 < kept < 1.0
        assert err <= 1e-2, err


def test_sparse_v_rejects_bad_arguments(fm, dev):
    cache = fm.KVCache.new_affine(1, 2, 256, 64, device=dev)
    q = torch.zeros(1, 4, 256, dtype=torch.bfloat16, device=dev)
    with pytest.raises(fm.FmoeError):
        cache.attend_sparse_v(q, 0.01, n_valid=8)  # affine storage
    cache = fm.KVCache(1, 2, 256, 64, device=dev)
    with pytest.raises(fm.FmoeError):
        cache.attend_sparse_v(q, 0.01, n_valid=65)  # beyond the ring
    with pytest.raises(fm.FmoeError):
        cache.attend_sparse_v(q, -1.0, n_valid=8)


# ---------------------------------------------------------------------------
# The gate inside the decoder layer (Gemma4DecoderLayer.sparse_v_tau,
# Gemma4Model.set_sparse_v_threshold = Model::set_sparse_v_threshold,
# src/model/mod.rs:367-372; decode only, gemma4_attention.rs:91-93).
#
# Tolerance: the whole layer within 2e-2 of the oracle's layer with the same tau
# (the layer tolerance of the dense decode tests).  tau sits mid-gap between two
# of the oracle's softmax weights near the weight below which the weights hold
# 15 % of the softmax mass (so the gate changes the output); the GPU's weights
# differ from the oracle's by bf16 rounding of q, so a weight close to tau may
# still fall on the other side: each such flip moves one head's output by about
# tau * |v|, well inside the tolerance.  With tau at the 15 %-mass weight the
# gate must move the layer's output by more than the GPU / oracle difference,
# so it is not a no-op.

def _layer_probs(orc, q, ck, n, Hkv, scale):
    """Softmax weights [T, Hq, n] of the oracle's rotated queries q [T, Hq, D]
    over the first n slots of ck [T, Hkv, cap, D] (float64)."""
    qf = orc.bf16_to_f32(q).astype(np.float64)
    kf = orc.bf16_to_f32(ck[:, :, :n]).astype(np.float64)
    R = qf.shape[1] // Hkv
    s = np.einsum("bhd,bhtd->bht", qf, np.repeat(kf, R, axis=1)) * scale
    s -= s.max(axis=2, keepdims=True)
    p = np.exp(s)
    return p / p.sum(axis=2, keepdims=True)


def _mass_target(p, frac):
    """The weight below which the pooled weights of all rows hold `frac` of the
    total mass (the softmax at these shapes is peaked: most weights are tiny)."""
    w = np.sort(p.ravel())
    c = np.cumsum(w)
    return float(w[min(int(np.searchsorted(c, frac * c[-1])), w.size - 1)])


def _widest_gap_tau(p, target):
    """The midpoint of the widest gap between weights within 0.7 .. 1.3 x target."""
    w = np.sort(p[(p > 0.7 * target) & (p < 1.3 * target)].ravel())
    if w.size < 2:
        return target
    i = int(np.argmax(np.diff(w)))
    return float(0.5 * (w[i] + w[i + 1]))


@pytest.mark.parametrize("target", ["mass", "uniform"])
@pytest.mark.parametrize("full,kv", [(False, "bf16"), (True, "bf16"), (False, "turbo3")])
def test_decoder_layer_sparse_v_matches_oracle(fm, orc, dev, full, kv, target):
    """target "mass": tau near the weight below which the weights hold 15 % of
    the softmax mass (the gate visibly moves the layer output); "uniform": tau
    near 1 / attended slots, the reference's typical small threshold (only the
    tail goes, which here carries little mass)."""
    from test_gpu_decoder import LAYER_TOL, oracle_cfg, oracle_weights
    from gpu_util import topk_sure

    cfg = dict(fm.GEMMA4_26B)
    T, cap, pos = 2, 512, 400
    for seed in (61, 1061, 2061, 3061):
        L = fm.Gemma4DecoderLayer.random(cfg, full, seed=seed + full, device=dev)
        cache = fm.KVCache(T, L.num_kv_heads, L.head_dim, cap, turbo_bits=3 if kv == "turbo3" else 0, device=dev)
        g = torch.Generator(device=dev).manual_seed(seed)
        cache.update(torch.randn(T, L.num_kv_heads, pos, L.head_dim, generator=g, device=dev).to(torch.bfloat16),
                     torch.randn(T, L.num_kv_heads, pos, L.head_dim, generator=g, device=dev).to(torch.bfloat16))
        x = torch.randn(T, cfg["hidden"], generator=g, device=dev).to(torch.bfloat16)
        x_in = to_np_bf16(x)
        a = cache.arrays()
        ck0, cv0 = to_np_bf16(a["k"]).copy(), to_np_bf16(a["v"]).copy()
        W = oracle_weights(L)
        ocfg = oracle_cfg(L, cfg)
        ocfg["turbo_bits"] = cache.turbo_bits
        ck, cv = ck0.copy(), cv0.copy()
        x_dense, q = orc.decoder_layer(x_in, W, ck, cv, pos, ocfg)
        if not topk_sure(ocfg["_router_logits"], L.top_k).all():
            continue
        p = _layer_probs(orc, q, ck, pos + 1, L.num_kv_heads, L.attn_scale)
        tau = _widest_gap_tau(p, _mass_target(p, 0.15) if target == "mass" else 1.0 / (pos + 1))
        gcfg = dict(ocfg, sparse_v_tau=tau)
        x_gate, _ = orc.decoder_layer(x_in, W, ck0.copy(), cv0.copy(), pos, gcfg)
        if not topk_sure(gcfg["_router_logits"], L.top_k).all():
            continue
        L.sparse_v_tau = tau
        L._c = None
        ws = torch.zeros(L.workspace_bytes(T, cache), dtype=torch.uint8, device=dev)
        L.forward(x, cache, pos, ws)
        torch.cuda.synchronize()
        got = orc.bf16_to_f32(to_np_bf16(x))
        err = max_rel_err(got, orc.bf16_to_f32(x_gate))
        moved = max_rel_err(orc.bf16_to_f32(x_gate), orc.bf16_to_f32(x_dense))
        kept = float((p >= tau).mean())
        print(f"tau {tau:.3e}: {kept:.3f} of the weights kept; layer err {err:.4f}, gate moved the output {moved:.4f}")
        assert cache.status() == 0
        assert 0.0 < kept < 1.0
        assert err <= LAYER_TOL, err
        if target == "mass":
            assert moved > err, (moved, err)
        return
    pytest.skip("router logits tie within 1e-3 at the top-k boundary for every seed tried")


def test_sparse_v_decode_step_graph_replay(fm, dev):
    """Model-level threshold: eager steps and CUDA-graph replays (attended slot
    count read on the device) give the same tokens and logits; the gate changes
    the logits; the single-kernel step refuses a gated model."""
    cfg = dict(fm.GEMMA4_26B, vocab=4096, full_every=2)
    ctx = 300
    m1 = fm.Gemma4Model.random(cfg, batch=1, max_positions=512, seed=13, device=dev, n_layers=2)
    m2 = fm.Gemma4Model(cfg, m1.embed, m1.layers, m1.final_norm, 1, 512, device=dev)
    g = torch.Generator(device=dev).manual_seed(14)
    for L, c1, c2 in zip(m1.layers, m1.caches, m2.caches):
        kv = torch.randn(2, 1, L.num_kv_heads, ctx, L.head_dim, generator=g, device=dev).to(torch.bfloat16)
        c1.update(kv[0], kv[1])
        c2.update(kv[0], kv[1])
    m1.ids.fill_(9)
    m1.set_position(ctx)
    m1.decode_step()
    dense = m1.logits.clone()
    m1.set_sparse_v_threshold(2e-3)  # the layers are shared with m2
    m1.ids.fill_(9)
    m1.set_position(ctx)  # rewrites the same slot
    out_eager = []
    for _ in range(3):
        out_eager.append((m1.decode_step().clone(), m1.logits.clone()))
    assert not torch.equal(out_eager[0][1], dense)
    m2.ids.fill_(9)
    m2.set_position(ctx)
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        graph = torch.cuda.CUDAGraph()
        ids0, pos0 = m2.ids.clone(), m2.pos_dev.clone()
        m2.decode_step(device_pos=True)
        torch.cuda.synchronize()
        m2.ids.copy_(ids0)
        m2.pos_dev.copy_(pos0)
        torch.cuda.synchronize()
        with torch.cuda.graph(graph, stream=s):
            m2.decode_step(device_pos=True)
    torch.cuda.current_stream().wait_stream(s)
    for step in range(3):
        graph.replay()
        torch.cuda.synchronize()
        assert torch.equal(m2.ids, out_eager[step][0])
        assert torch.equal(m2.logits, out_eager[step][1])
    del graph
    with pytest.raises(fm.FmoeError):
        m1.decode_step_fused()
    m1.set_sparse_v_threshold(0.0)
