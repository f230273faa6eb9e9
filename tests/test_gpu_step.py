"""GPU parity: the whole decode step as one persistent kernel (fmoe_decode_step).

Pinned against the oracle's composition of the reference's step for one
sequence: embedding row * sqrt(hidden) (src/model/mod.rs:145-160), one
DecoderLayer::forward_gemma4 (mod.rs:67-119) and the final norm + tied
lm_head + softcap + argmax (mod.rs:254, 336-362); and against the layered
path (fmoe_decoder_layer_forward per layer) on a two-layer model.

Tolerance (max |gpu - oracle| / max |oracle|): 2e-2 on the logits, the bound
the single-layer test holds a layer's output to (a layer moves by 0.9-1.6 %
under +-1 bf16 ulp of input noise; the lm_head adds one more bf16-rounded
GEMV).  The next token must match wherever the oracle's top-2 logits are more
than 1e-3 (relative) apart.  A case whose router logits tie within 1e-3 at
the top-k boundary is skipped (the routed experts then legitimately differ).
"""
import numpy as np
import pytest
import torch

from gpu_util import max_rel_err, to_np_bf16, to_np_u32, topk_sure
from test_gpu_decoder import oracle_cfg, oracle_weights

pytestmark = pytest.mark.gpu
TOL = 2e-2


def _model(fm, dev, full, ctx, seed, vocab=4096, n_layers=1, full_every=None):
    cfg = dict(fm.GEMMA4_26B, vocab=vocab, full_every=full_every or (1 if full else 5))
    m = fm.Gemma4Model.random(cfg, batch=1, max_positions=max(ctx, 1024) + 64, seed=seed, device=dev,
                              n_layers=n_layers)
    g = torch.Generator(device=dev).manual_seed(seed + 1)
    for L, c in zip(m.layers, m.caches):
        for p0 in range(0, ctx, 256):
            n = min(256, ctx - p0)
            kv = torch.randn(2, 1, L.num_kv_heads, n, L.head_dim, generator=g, device=dev).to(torch.bfloat16)
            c.update(kv[0], kv[1])
    return cfg, m


def _embed_row(orc, m, tok):
    e = m.embed
    row = orc.dequantize(to_np_u32(e.weight[tok:tok + 1]), to_np_bf16(e.scales[tok:tok + 1]),
                         to_np_bf16(e.biases[tok:tok + 1]), e.in_features, e.bits)
    es = orc.bf16_to_f32(orc.f32_to_bf16(np.float32([m._emb_scale])))[0]
    return orc.f32_to_bf16(orc.bf16_to_f32(row) * es)  # dequantize returns bf16(fma(s, q, b)) bits


@pytest.mark.parametrize("full,ctx", [(False, 700), (False, 1100), (True, 700), (False, 0), (True, 37)])
def test_fused_step_matches_oracle(fm, orc, dev, full, ctx):
    cfg, m = _model(fm, dev, full, ctx, seed=71 + ctx + full)
    L, cache = m.layers[0], m.caches[0]
    tok = 123
    m.ids.fill_(tok)
    m.set_position(ctx)
    a = cache.arrays()
    ck, cv = to_np_bf16(a["k"]).copy(), to_np_bf16(a["v"]).copy()
    m.decode_step_fused()
    torch.cuda.synchronize()
    assert m.fused_status() == 0
    assert int(m.pos_dev[0]) == ctx + 1
    x0 = _embed_row(orc, m, tok)
    ocfg = oracle_cfg(L, cfg)
    x1, _ = orc.decoder_layer(x0, oracle_weights(L), ck, cv, ctx, ocfg)
    if not topk_sure(ocfg["_router_logits"], L.top_k).all():
        pytest.skip("router logits tie within 1e-3 at the top-k boundary")
    e = m.embed
    want, want_ids = orc.lm_head(x1, (to_np_u32(e.weight), to_np_bf16(e.scales), to_np_bf16(e.biases), e.in_features,
                                      e.bits), to_np_bf16(m.final_norm), cfg["eps"], cfg["softcap"])
    got = m.logits.cpu().numpy()
    err = max_rel_err(got, want)
    assert err <= TOL, err
    # the appended K / V rows
    a = cache.arrays()
    slot = ctx % cache.capacity
    kerr = max_rel_err(orc.bf16_to_f32(to_np_bf16(a["k"][:, :, slot])), orc.bf16_to_f32(ck[:, :, slot]))
    verr = max_rel_err(orc.bf16_to_f32(to_np_bf16(a["v"][:, :, slot])), orc.bf16_to_f32(cv[:, :, slot]))
    assert kerr <= 1e-2 and verr <= 1e-2, (kerr, verr)
    srt = -np.sort(-want[0])
    if srt[0] - srt[1] > 1e-3 * abs(srt[0]):
        assert int(m.ids[0]) == int(want_ids[0])


def test_fused_step_matches_layered_two_layers(fm, dev):
    """A sliding and a full layer: the fused kernel and the per-layer path
    agree on the logits, the next token and the appended cache rows."""
    ctx = 900
    cfg, m1 = _model(fm, dev, False, ctx, seed=5, n_layers=2, full_every=2)
    m2 = fm.Gemma4Model(cfg, m1.embed, m1.layers, m1.final_norm, 1, max(ctx, 1024) + 64, device=dev)
    for c1, c2 in zip(m1.caches, m2.caches):
        a1, a2 = c1.arrays(), c2.arrays()
        a2["k"].copy_(a1["k"])
        a2["v"].copy_(a1["v"])
        c2._offset = c1._offset
    for mm in (m1, m2):
        mm.ids.fill_(77)
        mm.set_position(ctx)
    m1.decode_step()
    m2.decode_step_fused()
    torch.cuda.synchronize()
    assert m2.fused_status() == 0
    a, b = m1.logits.cpu().numpy(), m2.logits.cpu().numpy()
    assert max_rel_err(b, a) <= TOL
    srt = -np.sort(-a[0])
    if srt[0] - srt[1] > 1e-2 * abs(srt[0]):
        assert int(m1.ids[0]) == int(m2.ids[0])
    for c1, c2 in zip(m1.caches, m2.caches):
        slot = ctx % c1.capacity
        for key in ("k", "v"):
            r1 = c1.arrays()[key][:, :, slot].float().cpu().numpy()
            r2 = c2.arrays()[key][:, :, slot].float().cpu().numpy()
            assert max_rel_err(r2, r1) <= TOL


def test_fused_step_graph_replay(fm, dev):
    """The fused step captured in a CUDA graph: replays from the same state
    reproduce the eager step bit for bit; the position advances per replay."""
    ctx = 500
    cfg, m = _model(fm, dev, False, ctx, seed=9, n_layers=2, full_every=2)
    m.ids.fill_(5)
    m.set_position(ctx)
    m.decode_step_fused()
    torch.cuda.synchronize()
    ref_ids, ref_logits = m.ids.clone(), m.logits.clone()
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        graph = torch.cuda.CUDAGraph()
        m.ids.fill_(5)
        m.set_position(ctx)
        torch.cuda.synchronize()
        with torch.cuda.graph(graph, stream=s):
            m.decode_step_fused()
    torch.cuda.current_stream().wait_stream(s)
    for _ in range(2):
        m.ids.fill_(5)
        m.set_position(ctx)
        torch.cuda.synchronize()
        graph.replay()
        torch.cuda.synchronize()
        assert torch.equal(m.ids, ref_ids)
        assert torch.equal(m.logits, ref_logits)
        assert int(m.pos_dev[0]) == ctx + 1
    assert m.fused_status() == 0
    del graph


@pytest.mark.parametrize("kv", ["affine", "turbo3"])
@pytest.mark.parametrize("full", [False, True])
def test_layered_step_cache_modes_match_oracle(fm, orc, dev, kv, full):
    """Gemma4Model.decode_step (one fmoe_decoder_layer_forward per layer, then
    the lm_head) with the WHT-rotated affine K4 / V8 cache and with the
    reference's default TurboQuant-3 cache (src/main.rs:53, src/cache.rs:
    290-308), against the oracle's composition of the step on the same caches.
    Seeds whose router logits tie at the top-k boundary are passed over."""
    for seed in (91 + full, 191 + full, 291 + full, 391 + full):
        if _layered_step_case(fm, orc, dev, kv, full, seed):
            return
    pytest.skip("router logits tie within 1e-3 at the top-k boundary for every seed tried")


def _layered_step_case(fm, orc, dev, kv, full, seed):
    ctx = 700
    cfg = dict(fm.GEMMA4_26B, vocab=4096, full_every=1 if full else 5)
    m = fm.Gemma4Model.random(cfg, batch=1, max_positions=1024 + 64, seed=seed, device=dev, n_layers=1,
                              kv_mode=fm.KV_AFFINE if kv == "affine" else fm.KV_BF16,
                              turbo_bits=3 if kv == "turbo3" else 0)
    L, cache = m.layers[0], m.caches[0]
    g = torch.Generator(device=dev).manual_seed(seed + 1)
    for p0 in range(0, ctx, 256):
        n = min(256, ctx - p0)
        kvr = torch.randn(2, 1, L.num_kv_heads, n, L.head_dim, generator=g, device=dev).to(torch.bfloat16)
        cache.update(kvr[0], kvr[1])
    a = cache.arrays()
    ocfg = oracle_cfg(L, cfg)
    if kv == "affine":
        ck = (to_np_u32(a["k"]).copy(), to_np_bf16(a["k_scales"]).copy(), to_np_bf16(a["k_biases"]).copy())
        cv = (to_np_u32(a["v"]).copy(), to_np_bf16(a["v_scales"]).copy(), to_np_bf16(a["v_biases"]).copy())
        ocfg["kv_mode"] = "affine"
    else:
        ck, cv = to_np_bf16(a["k"]).copy(), to_np_bf16(a["v"]).copy()
        ocfg["turbo_bits"] = 3
    tok = 321
    m.ids.fill_(tok)
    m.set_position(ctx)
    m.decode_step()
    torch.cuda.synchronize()
    x1, _ = orc.decoder_layer(_embed_row(orc, m, tok), oracle_weights(L), ck, cv, ctx, ocfg)
    if not topk_sure(ocfg["_router_logits"], L.top_k).all():
        return False
    e = m.embed
    want, want_ids = orc.lm_head(x1, (to_np_u32(e.weight), to_np_bf16(e.scales), to_np_bf16(e.biases), e.in_features,
                                      e.bits), to_np_bf16(m.final_norm), cfg["eps"], cfg["softcap"])
    err = max_rel_err(m.logits.cpu().numpy(), want)
    assert err <= TOL, err
    srt = -np.sort(-want[0])
    if srt[0] - srt[1] > 1e-3 * abs(srt[0]):
        assert int(m.ids[0]) == int(want_ids[0])
    return True


@pytest.mark.parametrize("B,full_every,batched", [(32, 5, "1"), (32, 5, "0"), (20, 1, "1")])
def test_layered_step_batch32_matches_oracle(fm, orc, dev, monkeypatch, B, full_every, batched):
    """Decode at batch 32 (BASELINE config 4's batch), and a ragged batch of 20
    on a full-attention layer: batched "1" runs each layer as one call (the
    attention half per group of 8 inside the library, router / experts / dense
    MLP once over the batch); "0" as calls of 8 sequences on views of one cache.
    Every sequence's logits against the oracle's composition of the step for all
    tokens at once; sequences whose routing is a near tie at the top-k boundary
    are left out (at least half must remain)."""
    monkeypatch.setenv("FMOE_BATCHED_LAYER", batched)
    ctx, seed = 300, 511
    cfg = dict(fm.GEMMA4_26B, vocab=4096, full_every=full_every)
    m = fm.Gemma4Model.random(cfg, batch=B, max_positions=1024 + 64, seed=seed, device=dev, n_layers=1)
    assert len(m.groups) == (B + 7) // 8
    assert len(m.layer_groups) == (1 if batched == "1" else len(m.groups))
    L, cache = m.layers[0], m.caches[0]
    g = torch.Generator(device=dev).manual_seed(seed + 1)
    for p0 in range(0, ctx, 150):
        kvr = torch.randn(2, B, L.num_kv_heads, 150, L.head_dim, generator=g, device=dev).to(torch.bfloat16)
        cache.update(kvr[0], kvr[1])
    a = cache.arrays()
    ck, cv = to_np_bf16(a["k"]).copy(), to_np_bf16(a["v"]).copy()
    toks = torch.randint(0, cfg["vocab"], (B,), generator=g, device=dev, dtype=torch.int32)
    m.ids.copy_(toks)
    m.set_position(ctx)
    m.decode_step()
    torch.cuda.synchronize()
    x0 = np.concatenate([_embed_row(orc, m, int(t)) for t in toks.cpu()], 0)
    ocfg = oracle_cfg(L, cfg)
    x1, _ = orc.decoder_layer(x0, oracle_weights(L), ck, cv, ctx, ocfg)
    e = m.embed
    want, want_ids = orc.lm_head(x1, (to_np_u32(e.weight), to_np_bf16(e.scales), to_np_bf16(e.biases), e.in_features,
                                      e.bits), to_np_bf16(m.final_norm), cfg["eps"], cfg["softcap"])
    sure = topk_sure(ocfg["_router_logits"], L.top_k)
    assert sure.mean() >= 0.5, sure.mean()
    got = m.logits.cpu().numpy()
    for b in np.nonzero(sure)[0]:
        err = max_rel_err(got[b], want[b])
        assert err <= TOL, (b, err)
    # the appended rows of every sequence
    a = cache.arrays()
    kerr = max_rel_err(orc.bf16_to_f32(to_np_bf16(a["k"][:, :, ctx])), orc.bf16_to_f32(ck[:, :, ctx]))
    assert kerr <= 1e-2, kerr


def _replay_three(m, ids0, ctx):
    """Three CUDA-graph replays of decode_step (position on the device) from
    ids0 at ctx: [(ids, logits)] after each."""
    m.ids.copy_(ids0)
    m.set_position(ctx)
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        graph = torch.cuda.CUDAGraph()
        ids_c, pos_c = m.ids.clone(), m.pos_dev.clone()
        m.decode_step(device_pos=True)  # outside capture: library set-up; state restored below
        torch.cuda.synchronize()
        m.ids.copy_(ids_c)
        m.pos_dev.copy_(pos_c)
        torch.cuda.synchronize()
        with torch.cuda.graph(graph, stream=s, capture_error_mode="thread_local"):
            m.decode_step(device_pos=True)
    torch.cuda.current_stream().wait_stream(s)
    out = []
    for _ in range(3):
        graph.replay()
        torch.cuda.synchronize()
        out.append((m.ids.clone(), m.logits.clone()))
    del graph
    return out


def test_batched_layer_two_streams_identical_and_replayable(fm, dev, monkeypatch):
    """The batched layer runs the odd groups' attention half on a second stream
    with their own buffers (attention counters cleared per call, since their
    offset differs between sliding and full layers).  Over a sliding + full
    two-layer model at batch 32, one stream and two give identical tokens and
    logits, both in eager steps and in CUDA-graph replays.  (Eager steps and
    replays differ from each other in the last bits: a replay plans the
    split-KV attention for the whole ring, an eager step for the slots in use,
    so their partial softmax sums split the keys differently.)"""
    cfg = dict(fm.GEMMA4_26B, vocab=4096, full_every=2)
    B, ctx = 32, 300
    m = fm.Gemma4Model.random(cfg, batch=B, max_positions=512, seed=17, device=dev, n_layers=2)
    assert len(m.layer_groups) == 1
    g = torch.Generator(device=dev).manual_seed(18)
    for L, c in zip(m.layers, m.caches):
        kv = torch.randn(2, B, L.num_kv_heads, ctx, L.head_dim, generator=g, device=dev).to(torch.bfloat16)
        c.update(kv[0], kv[1])
    ids0 = torch.randint(0, cfg["vocab"], (B,), generator=g, device=dev, dtype=torch.int32)
    eager, replay = {}, {}
    for ns in ("1", "2"):
        monkeypatch.setenv("FMOE_BATCHED_STREAMS", ns)
        m.ids.copy_(ids0)
        m.set_position(ctx)  # the steps rewrite the same slots
        eager[ns] = [(m.decode_step().clone(), m.logits.clone()) for _ in range(3)]
        torch.cuda.synchronize()
        replay[ns] = _replay_three(m, ids0, ctx)
    assert m.status() == 0
    for runs in (eager, replay):
        for (a_ids, a_lg), (b_ids, b_lg) in zip(runs["1"], runs["2"]):
            assert torch.isfinite(a_lg).all()
            assert torch.equal(a_ids, b_ids)
            assert torch.equal(a_lg, b_lg)
