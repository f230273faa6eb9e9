"""GPU parity: prefill of a whole decoder layer (fmoe_decoder_layer_prefill) and
its new pieces against the oracle:

* the tensor-core quantised GEMM for many tokens (fmoe_qlinear with T > 8,
  fmoe_mlp_forward) — QuantizedLinear::forward / GeLUMLP::forward,
  src/model/mlp.rs:15-41;
* the causal / sliding prefill attention (fmoe_attn_prefill) over the ring's
  stored rows plus the new rows — src/model/mod.rs:682-753 masks,
  src/cache.rs:266-288, gemma4_attention.rs:95-104;
* a layer at the model's real shapes — src/model/mod.rs:67-119.

Tolerances (max |gpu - oracle| / max |oracle|): 1e-2 for a GEMM, the MLP and
attention (bf16 weights / P operands and bf16 outputs against the oracle's
fp32 / float64 arithmetic); 2e-2 for a layer's output and 1e-2 for the
appended K / V rows, as for the decode layer.  A layer's router input h2
comes out of attention over hundreds of tokens, so the GPU's and the oracle's
h2 differ by a few bf16 ulps here and there, and each router logit by up to
~1e-2: with hundreds of tokens some token's k-th and (k+1)-th experts then
swap, and its output row legitimately differs.  The layer tests therefore give
the router a logit bias of -8 on all but 8 experts (added before the bf16
rounding, as the router rule does): the routed set is the same for every
token on both sides, the weights among the 8 still come from the logits, and
every row is compared.  Over hundreds of tokens the largest per-token error
is an extreme of the same rounding noise the decode layer's 2e-2 bounds for
one or two tokens (Gemma-4's unscaled attention over RMS-normed q / k is
sharp: a 1-ulp difference can move which key dominates).  Each case therefore
measures that noise on the oracle itself — the same layer on x with +-1 bf16
ulp on 10 % of its elements — and holds the GPU's per-token error (max |diff|
of the token's row / max |oracle|) to 2e-2 or 1.5x the oracle's own, at the
median, the 99th percentile and the worst token.  With the TurboQuant round
trip a rotated value within rounding of a Lloyd-Max boundary may take the
neighbouring centroid, which moves its whole row: the stored rows' codes are
recovered and must equal the oracle's or be neighbours (at most 1 % differ),
and the oracle's layer then runs on the rows the GPU stored.
"""
import numpy as np
import pytest
import torch

from gpu_util import max_rel_err, to_np_bf16, to_np_u32, topk_sure
from test_gpu_decoder import oracle_cfg, oracle_weights

pytestmark = pytest.mark.gpu
TOL = 1e-2
LAYER_TOL = 2e-2


@pytest.mark.parametrize("bits,N,K,T", [(8, 4096, 2816, 9), (8, 4096, 2816, 512), (8, 2816, 4096, 200),
                                        (4, 2112, 2816, 64), (4, 2816, 2112, 333), (8, 1000, 704, 130),
                                        (4, 300, 512, 1000)])
def test_qlinear_many_tokens_matches_oracle(fm, orc, dev, bits, N, K, T):
    g = torch.Generator(device=dev).manual_seed(N + K + T + bits)
    q = fm.QuantizedLinear.from_float(torch.randn(N, K, generator=g, device=dev) * 0.02, bits)
    x = torch.randn(T, K, generator=g, device=dev).to(torch.bfloat16)
    y = q(x)
    torch.cuda.synchronize()
    want = orc.qmatmul(to_np_bf16(x), to_np_u32(q.weight), to_np_bf16(q.scales), to_np_bf16(q.biases), K, bits)
    err = max_rel_err(orc.bf16_to_f32(to_np_bf16(y)), want)
    assert err <= TOL, err


@pytest.mark.parametrize("T", [16, 300])
def test_mlp_forward_matches_oracle(fm, orc, dev, T):
    H, I = 2816, 2112
    g = torch.Generator(device=dev).manual_seed(T)
    gate, up, down = (fm.QuantizedLinear.from_float(torch.randn(o, i, generator=g, device=dev) * 0.02, 4)
                      for o, i in ((I, H), (I, H), (H, I)))
    x = torch.randn(T, H, generator=g, device=dev).to(torch.bfloat16)
    y = fm.mlp_forward(x, gate, up, down)
    torch.cuda.synchronize()
    ql = lambda w: (to_np_u32(w.weight), to_np_bf16(w.scales), to_np_bf16(w.biases), w.in_features, w.bits)
    want = orc.mlp(to_np_bf16(x), ql(gate), ql(up), ql(down))
    err = max_rel_err(orc.bf16_to_f32(to_np_bf16(y)), orc.bf16_to_f32(want))
    assert err <= TOL, err


ATTN_CASES = [
    # D, Hkv, Hq, cache capacity, window (0: full), pos0, T
    (256, 8, 16, 1024, 1024, 0, 512),     # sliding layer, first chunk of a prompt
    (256, 8, 16, 64, 64, 100, 300),       # ring wrapped, prompt longer than the window
    (256, 8, 16, 1024, 1024, 1500, 77),   # a later chunk: window spans ring and new rows
    (512, 2, 16, 2048, 0, 37, 200),       # full layer (K == V heads), causal
    (512, 2, 16, 2048, 0, 0, 1),
    (256, 8, 16, 64, 64, 5, 1),
]


@pytest.mark.parametrize("D,Hkv,Hq,cap,window,pos0,T", ATTN_CASES)
def test_attn_prefill_matches_oracle(fm, orc, dev, D, Hkv, Hq, cap, window, pos0, T):
    g = torch.Generator(device=dev).manual_seed(D + cap + pos0 + T)
    cache = fm.KVCache(1, Hkv, D, cap, window=window or None, device=dev)
    if pos0:
        cache.update(torch.randn(1, Hkv, pos0, D, generator=g, device=dev).to(torch.bfloat16),
                     torch.randn(1, Hkv, pos0, D, generator=g, device=dev).to(torch.bfloat16))
    q = (torch.randn(T, Hq, D, generator=g, device=dev) * 0.08).to(torch.bfloat16)
    kn = torch.randn(Hkv, T, D, generator=g, device=dev).to(torch.bfloat16)
    vn = torch.randn(Hkv, T, D, generator=g, device=dev).to(torch.bfloat16)
    out = cache.attend_prefill(q, kn, vn, pos0, window=window)
    torch.cuda.synchronize()
    a = cache.arrays()
    want = orc.attn_prefill_bf16(to_np_bf16(q), to_np_bf16(a["k"])[0], to_np_bf16(a["v"])[0], to_np_bf16(kn),
                                 to_np_bf16(vn), pos0, window, 1.0)
    err = max_rel_err(orc.bf16_to_f32(to_np_bf16(out)), want)
    assert err <= TOL, err


def _prefill_case(fm, orc, dev, full, T, pos0, window, turbo, seed):
    cfg = dict(fm.GEMMA4_26B)
    L = fm.Gemma4DecoderLayer.random(cfg, full, seed=seed, device=dev)
    keep = torch.randperm(cfg["experts"], generator=torch.Generator().manual_seed(seed))[:L.top_k]
    bias = torch.full((cfg["experts"],), -8.0)
    bias[keep] = 0.0
    L.router["logit_bias"] = bias.to(dev)
    L._c = None
    cap = window if window else 1024
    cache = fm.KVCache(1, L.num_kv_heads, L.head_dim, cap, window=window or None, turbo_bits=turbo, device=dev)
    g = torch.Generator(device=dev).manual_seed(seed)
    if pos0:
        cache.update(torch.randn(1, L.num_kv_heads, pos0, L.head_dim, generator=g, device=dev).to(torch.bfloat16),
                     torch.randn(1, L.num_kv_heads, pos0, L.head_dim, generator=g, device=dev).to(torch.bfloat16))
    x = torch.randn(T, cfg["hidden"], generator=g, device=dev).to(torch.bfloat16)
    x_in = to_np_bf16(x)
    a = cache.arrays()
    ck, cv = to_np_bf16(a["k"]).copy(), to_np_bf16(a["v"]).copy()
    ck0, cv0 = ck.copy(), cv.copy()
    ws = torch.zeros(L.prefill_workspace_bytes(T), dtype=torch.uint8, device=dev)
    L.prefill(x, cache, pos0, ws, window=window)
    torch.cuda.synchronize()
    assert fm.lib().fmoe_workspace_status(ws.data_ptr(), 0, None) == 0
    ocfg = oracle_cfg(L, cfg)
    ocfg["turbo_bits"] = turbo
    a = cache.arrays()
    rows = [(pos0 + t) % cap for t in range(max(0, T - cap), T)]
    gk, gv = to_np_bf16(a["k"])[0][:, rows], to_np_bf16(a["v"])[0][:, rows]  # [Hkv, T', D] as stored
    W = oracle_weights(L)
    nr = (gk, gv) if turbo and T <= cap else None
    xo, _ = orc.decoder_layer_prefill(x_in, W, ck, cv, pos0, window, ocfg, new_rows=nr)
    rng = np.random.default_rng(seed)
    xp = x_in.copy()
    hit = rng.random(xp.shape) < 0.1
    xp[hit] = (xp[hit].astype(np.int32) + rng.choice(np.array([-1, 1]), int(hit.sum()))).astype(np.uint16)
    xo_n, _ = orc.decoder_layer_prefill(xp, W, ck0, cv0, pos0, window, dict(ocfg), new_rows=nr)
    sure = topk_sure(ocfg["_router_logits"], L.top_k, margin=0.0)  # the k-th / (k+1)-th gap alone
    ok_k, ok_v = (orc.bf16_to_f32(r[:, max(0, T - cap):]) for r in ocfg["_new_rows"])
    row_k = np.abs(orc.bf16_to_f32(gk) - ok_k).max(2) / np.abs(ok_k).max()
    row_v = np.abs(orc.bf16_to_f32(gv) - ok_v).max(2) / np.abs(ok_v).max()
    got, want = orc.bf16_to_f32(to_np_bf16(x)), orc.bf16_to_f32(xo)
    scale = np.abs(want).max()
    tok_err = np.abs(got - want).max(axis=1) / scale
    tok_noise = np.abs(orc.bf16_to_f32(xo_n) - want).max(axis=1) / scale
    stats = {q: (float(np.percentile(tok_err, q)), float(np.percentile(tok_noise, q))) for q in (50, 99, 100)}
    print(f"layer prefill T={T} full={full} turbo={turbo}: token error / oracle noise at the median, p99, max: "
          + ", ".join(f"{e:.4f} / {n:.4f}" for e, n in stats.values())
          + f"; rows k {row_k.max():.4f} v {row_v.max():.4f}")
    assert sure.all(), sure.mean()
    if turbo:
        D = L.head_dim
        for pre, gpu in zip(ocfg["_pre_round_trip"], (gk, gv)):
            _turbo_codes_close(orc, pre.transpose(1, 0, 2).reshape(-1, D), gpu.reshape(-1, D), turbo)
    else:
        assert row_k.max() <= TOL and row_v.max() <= TOL, (row_k.max(), row_v.max())
    for q, (e, n) in stats.items():
        assert e <= max(LAYER_TOL, 1.5 * n), (q, e, n)


def _turbo_codes_close(orc, pre_bf16, got_bf16, bits):
    """The Lloyd-Max code of every rotated value of the stored rows equals the
    oracle's round trip of the same (pre-round-trip) rows or is its neighbour,
    and at most 1 % of the codes differ (src/cache.rs:94-129)."""
    D = pre_bf16.shape[1]
    _, idx_o, nrm = orc.turbo_round_trip(pre_bf16, bits)
    Hm = orc.hadamard(D).astype(np.float64)
    sg = orc.signs(D).astype(np.float64)
    cent, _ = orc.lloyd_max(bits)
    g = orc.bf16_to_f32(got_bf16).astype(np.float64)
    vals = sg * (g @ Hm) / nrm.astype(np.float64)[:, None] * np.sqrt(D)
    idx_g = np.abs(vals[:, :, None] - cent[None, None, :].astype(np.float64)).argmin(2)
    d = np.abs(idx_g - idx_o.astype(np.int64))
    print(f"  turbo codes differing: {np.mean(d > 0):.4f}, max step {int(d.max())}")
    assert d.max() <= 1 and np.mean(d > 0) <= 1e-2


@pytest.mark.parametrize("full,T,pos0,window,turbo", [
    (False, 512, 0, 1024, 0),     # sliding layer, first 512 prompt tokens
    (False, 300, 40, 128, 0),     # prompt longer than the window, ring already holding 40 positions
    (True, 300, 0, 0, 0),         # full layer (K == V, partial RoPE)
    (False, 64, 9, 1024, 3),      # TurboQuant-3 cache (the reference's default)
])
def test_decoder_layer_prefill_matches_oracle(fm, orc, dev, full, T, pos0, window, turbo):
    _prefill_case(fm, orc, dev, full, T, pos0, window, turbo, seed=71 + T + full)


def _affine_arrays(orc, cache):
    a = cache.arrays()
    k = (to_np_u32(a["k"]).copy(), to_np_bf16(a["k_scales"]).copy(), to_np_bf16(a["k_biases"]).copy())
    v = (to_np_u32(a["v"]).copy(), to_np_bf16(a["v_scales"]).copy(), to_np_bf16(a["v_biases"]).copy())
    return k, v


def _affine_rows_close(orc, got, want, slots, bits, D):
    """The appended rows of the rotated affine cache, dequantised.  Their inputs
    match the oracle's to ~1 bf16 ulp of the group's values, so a group's bf16
    scale and bias may move (every value then shifts a little with the same
    code) and a value near a code boundary may take the neighbouring code; at 8
    bits a step (range / 255) is itself about one such ulp.  Every value within
    1.1 steps plus two ulps of its group's largest value of the oracle's; at 4
    bits, where a step is coarse, at most 2 % of the values beyond half a step
    (a different code)."""
    def deq(arrs):
        q, s_, b_ = (x[0][:, slots].reshape(len(slots) * x.shape[1], -1) for x in arrs)
        return orc.bf16_to_f32(orc.dequantize(q, s_, b_, D, bits)), orc.bf16_to_f32(s_)
    g, _ = deq(got)
    w, sw = deq(want)
    step = np.repeat(np.abs(sw), 64, axis=1)
    gmax = np.repeat(np.abs(w).reshape(w.shape[0], -1, 64).max(axis=2), 64, axis=1)
    ulp = np.exp2(np.floor(np.log2(np.maximum(gmax, 1e-30))) - 7)
    d = np.abs(g - w)
    flips = float(np.mean(d > 0.5 * step + ulp))
    print(f"  affine {bits}-bit rows: max |diff| / (1.1 step + 2 ulp) "
          f"{float((d / (1.1 * step + 2 * ulp)).max()):.3f}, beyond half a step {flips:.4f}")
    assert (d <= 1.1 * step + 2 * ulp).all()
    if bits == 4:
        assert flips <= 0.02


def _prefill_case_affine(fm, orc, dev, full, T, pos0, window, seed):
    cfg = dict(fm.GEMMA4_26B)
    L = fm.Gemma4DecoderLayer.random(cfg, full, seed=seed, device=dev)
    keep = torch.randperm(cfg["experts"], generator=torch.Generator().manual_seed(seed))[:L.top_k]
    bias = torch.full((cfg["experts"],), -8.0)
    bias[keep] = 0.0
    L.router["logit_bias"] = bias.to(dev)
    L._c = None
    cap = window if window else 1024
    cache = fm.KVCache.new_affine(1, L.num_kv_heads, L.head_dim, cap, window=window or None, device=dev)
    g = torch.Generator(device=dev).manual_seed(seed)
    if pos0:
        cache.update(torch.randn(1, L.num_kv_heads, pos0, L.head_dim, generator=g, device=dev).to(torch.bfloat16),
                     torch.randn(1, L.num_kv_heads, pos0, L.head_dim, generator=g, device=dev).to(torch.bfloat16))
    x = torch.randn(T, cfg["hidden"], generator=g, device=dev).to(torch.bfloat16)
    x_in = to_np_bf16(x)
    ck, cv = _affine_arrays(orc, cache)
    ck0, cv0 = tuple(a.copy() for a in ck), tuple(a.copy() for a in cv)
    ws = torch.zeros(L.prefill_workspace_bytes(T), dtype=torch.uint8, device=dev)
    L.prefill(x, cache, pos0, ws, window=window)
    torch.cuda.synchronize()
    assert fm.lib().fmoe_workspace_status(ws.data_ptr(), 0, None) == 0
    ocfg = oracle_cfg(L, cfg)
    ocfg["kv_mode"] = "affine"
    W = oracle_weights(L)
    xo, _ = orc.decoder_layer_prefill(x_in, W, ck, cv, pos0, window, ocfg)
    rng = np.random.default_rng(seed)
    xp = x_in.copy()
    hit = rng.random(xp.shape) < 0.1
    xp[hit] = (xp[hit].astype(np.int32) + rng.choice(np.array([-1, 1]), int(hit.sum()))).astype(np.uint16)
    xo_n, _ = orc.decoder_layer_prefill(xp, W, ck0, cv0, pos0, window, dict(ocfg))
    assert topk_sure(ocfg["_router_logits"], L.top_k, margin=0.0).all()
    gk, gv = _affine_arrays(orc, cache)
    slots = [(pos0 + t) % cap for t in range(max(0, T - cap), T)]
    _affine_rows_close(orc, gk, ck, slots, 4, L.head_dim)
    _affine_rows_close(orc, gv, cv, slots, 8, L.head_dim)
    got, want = orc.bf16_to_f32(to_np_bf16(x)), orc.bf16_to_f32(xo)
    scale = np.abs(want).max()
    tok_err = np.abs(got - want).max(axis=1) / scale
    tok_noise = np.abs(orc.bf16_to_f32(xo_n) - want).max(axis=1) / scale
    stats = {q: (float(np.percentile(tok_err, q)), float(np.percentile(tok_noise, q))) for q in (50, 99, 100)}
    print(f"layer prefill (affine cache) T={T} full={full}: token error / oracle noise at the median, p99, max: "
          + ", ".join(f"{e:.4f} / {n:.4f}" for e, n in stats.values()))
    for q, (e, n) in stats.items():
        assert e <= max(LAYER_TOL, 1.5 * n), (q, e, n)


@pytest.mark.parametrize("full,T,pos0,window", [
    (False, 300, 40, 128),   # sliding: ring rows dequantised as they are read, prompt longer than the window
    (True, 64, 37, 0),       # full layer, head_dim 512
])
def test_decoder_layer_prefill_affine_cache_matches_oracle(fm, orc, dev, full, T, pos0, window):
    """The rotated affine K4 / V8 cache: queries and new rows rotated, the new
    rows through the cache's quantise / dequantise round trip, the stored rows
    dequantised in the attention tile loader, the output rotated back."""
    _prefill_case_affine(fm, orc, dev, full, T, pos0, window, seed=171 + T + full)


def test_prefill_then_decode_matches_token_by_token_decode(fm, dev):
    """A 2-layer model (one sliding layer with a window shorter than the prompt,
    one full layer): prefill of a 40-token prompt gives the same last-position
    logits as feeding the prompt one token at a time through the decode path,
    and the decode step after it (reading the rows the prefill appended) agrees
    as well."""
    cfg = dict(fm.GEMMA4_26B)
    cfg["window"] = 16
    cfg["full_every"] = 2
    prompt = torch.randint(0, cfg["vocab"], (40,), generator=torch.Generator().manual_seed(3)).to(torch.int32)
    a = fm.Gemma4Model.random(cfg, 1, 128, seed=5, device=dev, n_layers=2)
    a.prefill(prompt.to(dev))
    b = fm.Gemma4Model.random(cfg, 1, 128, seed=5, device=dev, n_layers=2)
    for t in range(40):
        b.ids.copy_(prompt[t:t + 1].to(dev))
        b.decode_step()
    torch.cuda.synchronize()
    assert a.pos == b.pos == 40
    err = (a.logits - b.logits).abs().max().item() / b.logits.abs().max().item()
    assert err <= 5e-2, err
    s = torch.sort(b.logits[0], descending=True).values
    if (s[0] - s[1]).item() > 0.05 * s[0].abs().item():  # a clear greedy choice
        assert int(a.ids[0]) == int(b.ids[0])
    b.ids.copy_(a.ids)  # the same next input on both
    a.decode_step()
    b.decode_step()
    torch.cuda.synchronize()
    err2 = (a.logits - b.logits).abs().max().item() / b.logits.abs().max().item()
    assert err2 <= 5e-2, err2
