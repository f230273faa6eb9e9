"""CPU tests of the oracle: known-answer tests restated from the reference's
plain-Rust code, MLX-affine packing order, routing renormalisation, and
regression against the committed fixtures in tests/golden/."""
import json
import os

import numpy as np
import pytest

GOLD = os.path.join(os.path.dirname(__file__), "golden")


def test_hadamard_orthonormal_and_sylvester(orc):
    # generate_hadamard, src/cache.rs:6-26
    for n in (2, 8, 256, 512):
        h = orc.hadamard(n)
        assert np.abs(h @ h.T - np.eye(n)).max() < 1e-5
        assert np.allclose(np.abs(h), 1 / np.sqrt(n))
        assert np.array_equal(h, h.T)
    h4 = orc.hadamard(4) * 2
    assert np.array_equal(h4, np.array([[1, 1, 1, 1], [1, -1, 1, -1], [1, 1, -1, -1], [1, -1, -1, 1]], np.float32))


def test_lcg_signs_match_pure_python(orc):
    # deterministic_signs(n, 42), src/cache.rs:29-43, build_rht seed cache.rs:49
    want = np.load(os.path.join(GOLD, "lcg_signs_seed42.npy"))
    assert np.array_equal(orc.signs(512, 42), want)
    assert set(np.unique(want)) == {-1.0, 1.0}


def test_lloyd_max_tables(orc):
    # src/cache.rs:67-89
    ref = json.load(open(os.path.join(GOLD, "lloyd_max.json")))
    for bits in (2, 3, 4):
        c, b = orc.lloyd_max(bits)
        assert np.allclose(c, ref[str(bits)]["centroids"], atol=0) and np.allclose(b, ref[str(bits)]["boundaries"], atol=0)
        assert len(c) == 2 ** bits and np.all(np.diff(c) > 0) and np.all(np.diff(b) > 0)
        assert np.all((b > c[:-1]) & (b < c[1:]))


def test_wht_butterfly_equals_matrix(orc):
    rng = np.random.default_rng(0)
    x = rng.standard_normal((5, 256)).astype(np.float32)
    h = orc.hadamard(256).astype(np.float64)
    assert np.abs(orc.wht_rows(x) - x.astype(np.float64) @ h).max() < 1e-5


def test_nibble_packing_order(orc):
    # MLX-affine 4-bit: 8 codes per uint32, element j at bits 4*(j%8)
    codes = np.arange(64) % 16
    word = np.zeros((1, 8), np.uint32)
    for j, c in enumerate(codes):
        word[0, j // 8] |= np.uint32(c) << np.uint32(4 * (j % 8))
    one = orc.f32_to_bf16(np.ones((1, 1), np.float32))
    zero = orc.f32_to_bf16(np.zeros((1, 1), np.float32))
    deq = orc.bf16_to_f32(orc.dequantize(word, one, zero, 64, 4))
    assert np.array_equal(deq[0], codes.astype(np.float32))
    # 8-bit: 4 per word, byte order
    word8 = np.array([[0x04030201] + [0] * 15], np.uint32)
    deq8 = orc.bf16_to_f32(orc.dequantize(word8, one, zero, 64, 8))
    assert np.array_equal(deq8[0, :5], [1, 2, 3, 4, 0])


@pytest.mark.parametrize("bits", [2, 3, 4, 5, 6, 8])
def test_quantize_roundtrip_error(orc, bits):
    rng = np.random.default_rng(bits)
    w = (rng.standard_normal((16, 256)) * 0.02).astype(np.float32)
    wq, s, b = orc.quantize(w, bits)
    deq = orc.bf16_to_f32(orc.dequantize(wq, s, b, 256, bits))
    sc = np.repeat(orc.bf16_to_f32(s), 64, axis=1)
    assert np.all(np.abs(deq - w) <= 0.5 * sc + 1e-3 * np.abs(w) + 2e-4)


def test_quantize_fixture_regression(orc):
    d = np.load(os.path.join(GOLD, "quant_small.npz"))
    for bits in (2, 4, 6, 8):
        wq, s, b = orc.quantize(d["w"], bits)
        assert np.array_equal(wq, d[f"wq{bits}"]) and np.array_equal(s, d[f"s{bits}"]) and np.array_equal(b, d[f"b{bits}"])
        assert np.array_equal(orc.dequantize(wq, s, b, 256, bits), d[f"deq{bits}"])


def test_qmatmul_matches_dequantized_matmul(orc):
    rng = np.random.default_rng(3)
    w = (rng.standard_normal((32, 128)) * 0.02).astype(np.float32)
    x = orc.f32_to_bf16(rng.standard_normal((3, 128)).astype(np.float32))
    for bits in (4, 8):
        wq, s, b = orc.quantize(w, bits)
        y = orc.qmatmul(x, wq, s, b, 128, bits)
        # exact dequantised weight in float64
        deq = np.zeros((32, 128))
        for r in range(32):
            for c in range(128):
                pos = c * bits
                q = (int(wq[r, pos // 32]) >> (pos % 32)) & ((1 << bits) - 1)
                deq[r, c] = float(orc.bf16_to_f32(s[r:r + 1, c // 64:c // 64 + 1])[0, 0]) * q + \
                    float(orc.bf16_to_f32(b[r:r + 1, c // 64:c // 64 + 1])[0, 0])
        ref = orc.bf16_to_f32(x).astype(np.float64) @ deq.T
        assert np.abs(y - ref).max() <= 1e-5 * np.abs(ref).max()


def test_router_renormalised_topk(orc):
    rng = np.random.default_rng(5)
    x = orc.f32_to_bf16(rng.standard_normal((4, 128)).astype(np.float32))
    wr = orc.f32_to_bf16((rng.standard_normal((16, 128)) * 0.1).astype(np.float32))
    ids, w, lg = orc.router(x, wr, 4)
    assert np.allclose(w.sum(1), 1.0, atol=1e-6)
    # ranking and softmax see the logits rounded to bf16, the router's output
    # dtype (moe.rs:318-330); stable argsort = ties to the lower id
    lb = orc.bf16_to_f32(orc.f32_to_bf16(lg))
    for t in range(4):
        order = np.argsort(-lb[t], kind="stable")[:4]
        assert np.array_equal(ids[t], order)
        p = np.exp(lb[t] - lb[t].max())
        p /= p.sum()
        assert np.allclose(w[t], p[ids[t]] / p[ids[t]].sum(), rtol=1e-5)
    # per-expert scale multiplies after renormalisation (moe.rs:341-345)
    pes = orc.f32_to_bf16(np.linspace(0.5, 2.0, 16).astype(np.float32))
    ids2, w2, _ = orc.router(x, wr, 4, per_expert_scale=pes)
    assert np.array_equal(ids, ids2)
    assert np.allclose(w2, w * orc.bf16_to_f32(pes)[ids], rtol=1e-6)


def test_router_tie_breaks_to_lower_id(orc):
    x = orc.f32_to_bf16(np.ones((1, 64), np.float32))
    wr = orc.f32_to_bf16(np.zeros((8, 64), np.float32))
    ids, w, _ = orc.router(x, wr, 3)
    assert np.array_equal(ids[0], [0, 1, 2]) and np.allclose(w, 1 / 3)


def test_moe_fixture_regression_and_one_hot(orc):
    d = np.load(os.path.join(GOLD, "moe_small.npz"))
    H, I, E, K, T = d["dims"]
    ids, w, lg = orc.router(d["x"], d["wr"], int(K))
    assert np.array_equal(ids, d["ids"]) and np.array_equal(w, d["weights"])
    y32, y16 = orc.moe_experts(d["x"], ids, w, d["buf"], int(d["stride"]), d["offsets"], int(H), int(I))
    assert np.array_equal(y16, d["y16"])
    # one-hot routing (k=1, weight 1): output is exactly that expert's MLP
    one = np.array([[3]] * int(T), np.int32)
    ya, _ = orc.moe_experts(d["x"], one, np.ones((int(T), 1), np.float32), d["buf"], int(d["stride"]), d["offsets"],
                            int(H), int(I))
    yb, _ = orc.moe_experts(d["x"], np.array([[3, 5]] * int(T), np.int32), np.array([[1.0, 0.0]] * int(T), np.float32),
                            d["buf"], int(d["stride"]), d["offsets"], int(H), int(I))
    assert np.array_equal(ya, yb)


def test_turbo_round_trip_fixture_and_properties(orc):
    d = np.load(os.path.join(GOLD, "turbo_small.npz"))
    out, idx, nrm = orc.turbo_round_trip(d["v"], 3)
    assert np.array_equal(out, d["out"]) and np.array_equal(idx, d["idx"])
    v = orc.bf16_to_f32(d["v"]).astype(np.float64)
    assert np.allclose(nrm, np.linalg.norm(v, axis=1), rtol=1e-6)
    assert idx.max() <= 7
    o = orc.bf16_to_f32(out).astype(np.float64)
    cos = (o * v).sum(1) / np.linalg.norm(o, axis=1) / np.linalg.norm(v, axis=1)
    assert np.all(cos > 0.95)  # 3-bit Lloyd-Max keeps ~98% of the direction


def test_kv_affine_is_rotated_quantisation(orc):
    rng = np.random.default_rng(9)
    v = orc.f32_to_bf16(rng.standard_normal((4, 256)).astype(np.float32))
    for bits in (4, 8):
        wq, s, b = orc.kv_quant_affine(v, bits)
        r = orc.wht_rows(orc.bf16_to_f32(v))
        wq2, s2, b2 = orc.quantize(r, bits)
        assert np.array_equal(wq, wq2) and np.array_equal(s, s2) and np.array_equal(b, b2)
