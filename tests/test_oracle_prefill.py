"""CPU checks of the prefill oracle (no GPU): the prefill attention of T new
tokens (src/model/mod.rs:682-753 masks over update_and_fetch's stored + new
rows, src/cache.rs:266-288) equals T decode-attention steps, each after
storing its token's row in the ring (the decode oracle, checked separately),
for sliding rings that wrap and for full caches."""
import numpy as np
import pytest

import oracle as orc


def _bf(x):
    return orc.f32_to_bf16(np.asarray(x, np.float32))


@pytest.mark.parametrize("D,Hkv,Hq,cap,window,pos0,T", [
    (256, 2, 4, 16, 16, 20, 7),    # sliding, ring already wrapped, window == capacity
    (256, 1, 2, 16, 16, 3, 21),    # sliding, prompt longer than the window
    (512, 1, 4, 64, 0, 5, 9),      # full causal
    (256, 2, 2, 32, 0, 0, 1),      # first token, nothing cached
])
def test_attn_prefill_equals_sequential_decode(D, Hkv, Hq, cap, window, pos0, T):
    rng = np.random.default_rng(D + Hkv + cap + pos0 + T)
    ring_k = _bf(rng.standard_normal((1, Hkv, cap, D)))
    ring_v = _bf(rng.standard_normal((1, Hkv, cap, D)))
    q = _bf(rng.standard_normal((T, Hq, D)) * 0.1)
    k_new = _bf(rng.standard_normal((Hkv, T, D)))
    v_new = _bf(rng.standard_normal((Hkv, T, D)))
    scale = 1.0
    got = orc.attn_prefill_bf16(q, ring_k[0], ring_v[0], k_new, v_new, pos0, window, scale)
    ck, cv = ring_k.copy(), ring_v.copy()
    for t in range(T):
        p = pos0 + t
        ck[0, :, p % cap] = k_new[:, t]
        cv[0, :, p % cap] = v_new[:, t]
        # a ring of `window` slots holds exactly the window; a full cache its prefix
        n = min(p + 1, cap)
        want = orc.attn_decode_bf16(q[t:t + 1], Hkv, cap, np.zeros(1, np.int32), np.full(1, n, np.int32), ck, cv,
                                    scale)
        np.testing.assert_allclose(got[t], want[0], rtol=2e-4, atol=2e-5)


def test_attn_prefill_masks_future_and_old_positions():
    """A key outside [p - window + 1, p] never contributes: setting those rows to
    huge values leaves the output unchanged."""
    rng = np.random.default_rng(7)
    D, Hkv, Hq, cap, window, pos0, T = 256, 1, 1, 8, 8, 12, 6
    ring_k = _bf(rng.standard_normal((Hkv, cap, D)))
    ring_v = _bf(rng.standard_normal((Hkv, cap, D)))
    q = _bf(rng.standard_normal((T, Hq, D)) * 0.1)
    k_new = _bf(rng.standard_normal((Hkv, T, D)))
    v_new = _bf(rng.standard_normal((Hkv, T, D)))
    base = orc.attn_prefill_bf16(q, ring_k, ring_v, k_new, v_new, pos0, window, 1.0)
    # token 0 (p = 12) must not see new rows 1.. (future); last token (p = 17)
    # must not see the ring row of position 12 - 8 + 1 = 5 .. 9 (out of its window)
    v2 = v_new.copy()
    v2[:, T - 1] = _bf(np.full((Hkv, D), 1e4))
    out = orc.attn_prefill_bf16(q, ring_k, ring_v, k_new, v2, pos0, window, 1.0)
    np.testing.assert_array_equal(out[:T - 1], base[:T - 1])
    rv = ring_v.copy()
    rv[:, 5 % cap] = _bf(np.full((Hkv, D), 1e4))  # position 5: only tokens at p <= 12 see it
    out = orc.attn_prefill_bf16(q, ring_k, rv, k_new, v_new, pos0, window, 1.0)
    np.testing.assert_array_equal(out[1:], base[1:])
    assert not np.allclose(out[0], base[0])


@pytest.mark.parametrize("D,Hkv,Hq,cap,window,pos0,T", [(256, 2, 4, 16, 16, 20, 7), (512, 1, 4, 64, 0, 5, 9)])
def test_attn_prefill_affine_equals_sequential_decode(D, Hkv, Hq, cap, window, pos0, T):
    """Over the rotated affine K4 / V8 cache: the prefill attention equals T
    decode-attention steps of the affine decode oracle, each after storing its
    token's codes (the prefill rounds the dequantised rows and the rotated
    query to bf16, the decode oracle keeps them wider: 1e-2)."""
    rng = np.random.default_rng(D + cap + T)
    rows = _bf(rng.standard_normal((Hkv, cap, D)))
    kq = tuple(a.reshape(1, Hkv, cap, -1) for a in orc.kv_quant_affine(rows, 4))
    vq = tuple(a.reshape(1, Hkv, cap, -1) for a in orc.kv_quant_affine(_bf(rng.standard_normal((Hkv, cap, D))), 8))
    q = _bf(rng.standard_normal((T, Hq, D)) * 0.1)
    k_new = _bf(rng.standard_normal((Hkv, T, D)))
    v_new = _bf(rng.standard_normal((Hkv, T, D)))
    got, kc, vc = orc.attn_prefill_affine(q, tuple(a[0] for a in kq), tuple(a[0] for a in vq), k_new, v_new, pos0,
                                          window, 1.0)
    ck, cv = tuple(a.copy() for a in kq), tuple(a.copy() for a in vq)
    for t in range(T):
        p = pos0 + t
        for arr, new in zip(ck + cv, kc + vc):
            arr[0, :, p % cap] = new[:, t]
        n = min(p + 1, cap)
        want = orc.attn_decode_affine(q[t:t + 1], Hkv, cap, np.zeros(1, np.int32), np.full(1, n, np.int32), *ck, 4,
                                      *cv, 8, 1.0)
        err = np.abs(got[t] - want[0]).max() / np.abs(want[0]).max()
        assert err <= 1e-2, (t, err)
