"""GPU parity: Gemma-4 decoder layer (decode step) and the tied 6-bit lm_head
against the oracle's composition of the reference's layer
(src/model/mod.rs:67-119, gemma4_attention.rs:36-112, mlp.rs:28-41,
moe.rs:315-470, mod.rs:336-362), at the model's real shapes.

Tolerances (max |gpu - oracle| / max |oracle|): 1e-2 for the new K / V cache
rows and the lm_head logits; 2e-2 for a whole layer's output.  A layer chains
~15 bf16-rounded tensors (a bf16 residual stream, scale-1.0 attention over
RMS-normalised q / k), and its output moves by 0.9-1.6 % under +-1-ulp noise
on 10 % of its input with unchanged routing (measured on the oracle alone at
these shapes), so 1e-2 is below the layer's own rounding noise; its
components are held to 1e-2 in their own tests.  A layer's MoE output depends
on the routed ids, so a seed whose router logits put the k-th and (k+1)-th
expert within 1e-3 of each other (the benchmark's tie rule) is passed over
for the next one.
"""
import numpy as np
import pytest
import torch

from gpu_util import max_rel_err, to_np_bf16, to_np_u32, topk_sure

pytestmark = pytest.mark.gpu
TOL = 1e-2
LAYER_TOL = 2e-2


def _ql(q):
    return (to_np_u32(q.weight), to_np_bf16(q.scales), to_np_bf16(q.biases), q.in_features, q.bits)


def oracle_weights(L):
    r = L.router
    return {
        "q": _ql(L.q_proj), "k": _ql(L.k_proj), "v": None if L.k_eq_v else _ql(L.v_proj), "o": _ql(L.o_proj),
        "q_norm": to_np_bf16(L.q_norm), "k_norm": to_np_bf16(L.k_norm),
        "input_norm": to_np_bf16(L.norms["input"]), "post_attn_norm": to_np_bf16(L.norms["post_attn"]),
        "pre_ff_norm": to_np_bf16(L.norms["pre_ff"]), "post_ff_norm_1": to_np_bf16(L.norms["post_ff_1"]),
        "pre_ff_norm_2": to_np_bf16(L.norms["pre_ff_2"]), "post_ff_norm_2": to_np_bf16(L.norms["post_ff_2"]),
        "post_ff_norm": to_np_bf16(L.norms["post_ff"]),
        "gate": _ql(L.mlp[0]), "up": _ql(L.mlp[1]), "down": _ql(L.mlp[2]),
        "router": (to_np_bf16(r["proj"].weight), 16, to_np_bf16(r["router_scale"]), to_np_bf16(r["per_expert_scale"]),
                   r["root_size"]),
        "experts": (L.experts.buf.cpu().numpy(), L.experts.stride, L.experts.offsets),
        "logit_bias": None if r.get("logit_bias") is None else r["logit_bias"].float().cpu().numpy(),
    }


def oracle_cfg(L, cfg):
    return {"heads": L.num_heads, "kv_heads": L.num_kv_heads, "head_dim": L.head_dim, "rope_dims": L.rope_dims,
            "rope_theta": L.rope_theta, "eps": L.eps, "k_eq_v": L.k_eq_v, "scalar": L.layer_scalar,
            "attn_scale": L.attn_scale, "top_k": L.top_k, "inter_expert": cfg["expert_inter"]}


LAYER_CASES = [(full, T, "bf16", path) for path in ("ops", "stream") for full in (False, True) for T in (1, 2)] + \
    [(full, 2, kv, path) for path in ("ops", "stream") for full in (False, True) for kv in ("turbo3", "affine")]


@pytest.mark.parametrize("full,T,kv,path", LAYER_CASES)
def test_decoder_layer_matches_oracle(fm, orc, dev, monkeypatch, full, T, kv, path):
    """Both decode paths (FMOE_DECODE_PATH: the per-op kernels and the
    streaming six-launch layer) and the three cache kinds: bf16, bf16 with the
    TurboQuant-3 round trip on append, WHT-rotated affine K4 / V8."""
    monkeypatch.setenv("FMOE_DECODE_PATH", path)
    for seed in (31 + 7 * T + full, 1031 + 7 * T + full, 2031 + 7 * T + full, 3031 + 7 * T + full):
        if _layer_case(fm, orc, dev, full, T, kv, seed):
            return
    pytest.skip("router logits tie within 1e-3 at the top-k boundary for every seed tried")


def _layer_case(fm, orc, dev, full, T, kv, seed):
    """One seeded layer vs the oracle; False when the router's top-k boundary
    is a near tie (the routed experts may then legitimately differ)."""
    cfg = dict(fm.GEMMA4_26B)
    L = fm.Gemma4DecoderLayer.random(cfg, full, seed=seed, device=dev)
    cap = 64
    if kv == "affine":
        cache = fm.KVCache.new_affine(T, L.num_kv_heads, L.head_dim, cap, device=dev)
    else:
        cache = fm.KVCache(T, L.num_kv_heads, L.head_dim, cap, turbo_bits=3 if kv == "turbo3" else 0, device=dev)
    g = torch.Generator(device=dev).manual_seed(5 + T)
    pos = 5
    cache.update(torch.randn(T, L.num_kv_heads, pos, L.head_dim, generator=g, device=dev).to(torch.bfloat16),
                 torch.randn(T, L.num_kv_heads, pos, L.head_dim, generator=g, device=dev).to(torch.bfloat16))
    x = torch.randn(T, cfg["hidden"], generator=g, device=dev).to(torch.bfloat16)
    x_in = to_np_bf16(x)
    ws = torch.zeros(L.workspace_bytes(T, cache), dtype=torch.uint8, device=dev)
    a = cache.arrays()
    ocfg = oracle_cfg(L, cfg)
    if kv == "affine":
        ck = tuple(f(a[n]).copy() for f, n in ((to_np_u32, "k"), (to_np_bf16, "k_scales"), (to_np_bf16, "k_biases")))
        cv = tuple(f(a[n]).copy() for f, n in ((to_np_u32, "v"), (to_np_bf16, "v_scales"), (to_np_bf16, "v_biases")))
        ocfg["kv_mode"] = "affine"
    else:
        ck, cv = to_np_bf16(a["k"]).copy(), to_np_bf16(a["v"]).copy()
        ocfg["turbo_bits"] = cache.turbo_bits
    L.forward(x, cache, pos, ws)
    torch.cuda.synchronize()
    xo, _ = orc.decoder_layer(x_in, oracle_weights(L), ck, cv, pos, ocfg)
    if not topk_sure(ocfg["_router_logits"], L.top_k).all():
        return False
    a = cache.arrays()
    if kv == "affine":
        # The new rows are quantised from k / v that match the oracle's to
        # ~1 bf16 ulp; where a rotated value sits on a code boundary its code
        # moves by one step (1/15 of the group's range at 4 bits), so the rows
        # are compared dequantised: every element within one step of the
        # oracle's, and at most 2 % of them off by more than a bf16 ulp.
        _affine_close(orc, a, ck, "k", 4, pos)
        _affine_close(orc, a, cv, "v", 8, pos)
        kerr = verr = 0.0
    else:
        kerr = max_rel_err(orc.bf16_to_f32(to_np_bf16(a["k"][:, :, pos])), orc.bf16_to_f32(ck[:, :, pos]))
        verr = max_rel_err(orc.bf16_to_f32(to_np_bf16(a["v"][:, :, pos])), orc.bf16_to_f32(cv[:, :, pos]))
    got, want = orc.bf16_to_f32(to_np_bf16(x)), orc.bf16_to_f32(xo)
    err = max_rel_err(got, want)
    ulp = np.exp2(np.floor(np.log2(np.maximum(np.abs(want), 1e-30))) - 7)
    d_ulp = np.abs(got - want) / ulp
    diag = (f"max rel err {err:.4f}; max |diff| {np.abs(got - want).max():.4f} at |ref| "
            f"{np.abs(want).flat[np.argmax(np.abs(got - want))]:.3f}; elements > 1 bf16 ulp: "
            f"{int((d_ulp > 1.01).sum())} of {d_ulp.size}; max {d_ulp.max():.1f} ulp")
    print(diag)
    assert cache.status() == 0
    assert kerr <= TOL and verr <= TOL, (kerr, verr)
    assert err <= LAYER_TOL, diag
    return True


def _deq_np(orc, arrs, bits, pos):
    q, s, b = (x[:, :, pos] for x in arrs)
    D = q.shape[-1] * 32 // bits
    return orc.bf16_to_f32(orc.dequantize(q.reshape(-1, q.shape[-1]), s.reshape(-1, s.shape[-1]),
                                          b.reshape(-1, b.shape[-1]), D, bits))


def _affine_close(orc, a, want_arrs, name, bits, pos):
    got_arrs = (to_np_u32(a[name]), to_np_bf16(a[name + "_scales"]), to_np_bf16(a[name + "_biases"]))
    got, want = _deq_np(orc, got_arrs, bits, pos), _deq_np(orc, want_arrs, bits, pos)
    step = np.repeat(np.abs(orc.bf16_to_f32(want_arrs[1][:, :, pos].reshape(got.shape[0], -1))), 64, axis=1)
    ulp = np.exp2(np.floor(np.log2(np.maximum(np.abs(want), 1e-30))) - 7)
    d = np.abs(got - want)
    assert (d <= 1.01 * step + 2 * ulp).all(), (name, float((d / step).max()))
    assert (d > 2 * ulp).mean() <= 0.02, (name, float((d > 2 * ulp).mean()))


def test_lm_head_matches_oracle(fm, orc, dev):
    H, V, T = 2816, 8192, 2
    g = torch.Generator(device=dev).manual_seed(3)
    emb = fm.QuantizedLinear.from_float(torch.randn(V, H, generator=g, device=dev) * 0.02, 6)
    fnorm = (1.0 + 0.1 * torch.randn(H, generator=g, device=dev)).to(torch.bfloat16)
    x = (4.0 * torch.randn(T, H, generator=g, device=dev)).to(torch.bfloat16)
    import ctypes
    logits = torch.empty(T, V, dtype=torch.float32, device=dev)
    ids = torch.empty(T, dtype=torch.int32, device=dev)
    ws = torch.zeros(fm.lib().fmoe_lm_head_workspace_bytes(T), dtype=torch.uint8, device=dev)
    c = emb.cstruct()
    fm.check(fm.lib().fmoe_lm_head(ctypes.byref(c), fnorm.data_ptr(), 1e-6, x.data_ptr(), T, 30.0, logits.data_ptr(),
                                   ids.data_ptr(), None, ws.data_ptr(), ws.numel(), torch.cuda.current_stream().cuda_stream))
    torch.cuda.synchronize()
    want, want_ids = orc.lm_head(to_np_bf16(x), _ql(emb), to_np_bf16(fnorm), 1e-6, 30.0)
    got = logits.cpu().numpy()
    assert max_rel_err(got, want) <= TOL
    srt = -np.sort(-want, axis=1)
    for t in range(T):
        if srt[t, 0] - srt[t, 1] > 1e-3 * abs(srt[t, 0]):
            assert int(ids[t]) == int(want_ids[t])


@pytest.mark.parametrize("out_f,in_f,bits,T", [(8192, 2816, 8, 1), (2816, 4096, 8, 3), (4224, 2816, 4, 1),
                                               (2816, 2112, 4, 8), (4096, 2816, 6, 2)])
def test_tiled_weights_give_identical_gemv(fm, dev, out_f, in_f, bits, T):
    """The tile layout only changes how the weights are staged: bit-identical
    outputs, except where the standalone call accumulates column chunks with
    atomics (K = 4096 at 8 bits: sums in arrival order), there within 1e-2."""
    g = torch.Generator(device=dev).manual_seed(out_f + bits)
    w = torch.randn(out_f, in_f, generator=g, device=dev) * 0.02
    a = fm.QuantizedLinear.from_float(w, bits)
    split = 16 * in_f * bits // 8 > 48 * 1024  # needs column chunks: accumulating output
    b = fm.QuantizedLinear(a.weight, a.scales, a.biases, bits, 64, in_features=in_f).tile(accumulate=split)
    x = torch.randn(T, in_f, generator=g, device=dev).to(torch.bfloat16)
    ya, yb = a.forward(x), b.forward(x)
    if split:
        assert max_rel_err(yb.float().cpu().numpy(), ya.float().cpu().numpy()) <= 1e-2
    else:
        assert torch.equal(ya, yb)


def test_decoder_tiled_weights_identical(fm, dev):
    cfg = dict(fm.GEMMA4_26B, vocab=4096, full_every=2)
    ctx = 300
    m1 = fm.Gemma4Model.random(cfg, batch=1, max_positions=1024, seed=31, device=dev, n_layers=2)
    g = torch.Generator(device=dev).manual_seed(32)
    kvs = []
    for L, c in zip(m1.layers, m1.caches):
        kv = torch.randn(2, 1, L.num_kv_heads, ctx, L.head_dim, generator=g, device=dev).to(torch.bfloat16)
        c.update(kv[0], kv[1])
        kvs.append(kv)
    m1.ids.fill_(9)
    m1.set_position(ctx)
    want = [(m1.decode_step().clone(), m1.logits.clone()) for _ in range(2)]
    m2 = fm.Gemma4Model(cfg, m1.embed, m1.layers, m1.final_norm, 1, 1024, device=dev).tile_weights()
    for kv, c in zip(kvs, m2.caches):
        c.update(kv[0], kv[1])
    m2.ids.fill_(9)
    m2.set_position(ctx)
    for ids, lg in want:
        assert torch.equal(m2.decode_step(), ids)
        assert torch.equal(m2.logits, lg)


@pytest.mark.parametrize("path", ["ops", "stream"])
def test_decode_step_graph_replay_is_deterministic(fm, dev, monkeypatch, path):
    """Eager steps and CUDA-graph replays (position on the device) give the same
    tokens and logits; the position advances once per step.  700 cached
    positions: both layer types run split-KV attention with the in-kernel merge,
    sharing one workspace.  Both decode paths: the streaming layer's pieces are
    claimed by whichever CTA arrives last, yet every sum has a fixed order."""
    monkeypatch.setenv("FMOE_DECODE_PATH", path)
    cfg = dict(fm.GEMMA4_26B, vocab=4096, full_every=2)
    ctx = 700
    m1 = fm.Gemma4Model.random(cfg, batch=1, max_positions=1024, seed=11, device=dev, n_layers=2)
    m2 = fm.Gemma4Model(cfg, m1.embed, m1.layers, m1.final_norm, 1, 1024, device=dev)
    g = torch.Generator(device=dev).manual_seed(12)
    for L, c1, c2 in zip(m1.layers, m1.caches, m2.caches):
        kv = torch.randn(2, 1, L.num_kv_heads, ctx, L.head_dim, generator=g, device=dev).to(torch.bfloat16)
        c1.update(kv[0], kv[1])
        c2.update(kv[0], kv[1])
    m1.ids.fill_(7)
    m1.set_position(ctx)
    out_eager = []
    for _ in range(3):
        out_eager.append((m1.decode_step().clone(), m1.logits.clone()))
    assert all(torch.isfinite(lg).all() for _, lg in out_eager)
    m2.ids.fill_(7)
    m2.set_position(ctx)
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        graph = torch.cuda.CUDAGraph()
        # one call outside capture (library attribute setup); it writes the same
        # cache slot the first replay rewrites, then the state is restored
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
    assert int(m2.pos_dev[0]) == ctx + 3
    del graph
