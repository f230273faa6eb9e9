"""CPU check of the oracle's sparse-V gate (no GPU): orc.attn_decode_bf16 with
tau against a float64 restatement of the reference's sparse_v_attention
(src/model/gemma4_attention.rs:196-234): softmax(q . K^T) over the attended
slots, weights below tau replaced by zero (the others keep their values, no
renormalisation), then weights . V, the query heads of a group sharing their
kv head.  Gemma 4 applies no extra score scale there (its SDPA scale is 1.0).

tau is placed mid-gap between two of the float64 weights, so the oracle's own
rounding cannot move a weight across it; outputs agree to 1e-4 of max |out|.
"""
import numpy as np
import pytest

import oracle as orc


def _bf(x):
    return orc.f32_to_bf16(np.asarray(x, np.float32))


def _reference(q, k, v, n, Hkv, tau):
    qf = orc.bf16_to_f32(q).astype(np.float64)           # [B, Hq, D]
    kf = orc.bf16_to_f32(k[:, :, :n]).astype(np.float64)  # [B, Hkv, n, D]
    vf = orc.bf16_to_f32(v[:, :, :n]).astype(np.float64)
    R = qf.shape[1] // Hkv
    s = np.einsum("bhd,bhtd->bht", qf, np.repeat(kf, R, axis=1))
    s -= s.max(axis=2, keepdims=True)
    w = np.exp(s)
    w /= w.sum(axis=2, keepdims=True)
    gated = np.where(w >= tau, w, 0.0)
    return np.einsum("bht,bhtd->bhd", gated, np.repeat(vf, R, axis=1)), w


@pytest.mark.parametrize("B,Hkv,Hq,D,cap,n", [(1, 2, 4, 256, 64, 50), (2, 1, 8, 512, 32, 32)])
def test_oracle_sparse_v_matches_reference_restatement(B, Hkv, Hq, D, cap, n):
    rng = np.random.default_rng(B + Hkv + D + n)
    q = _bf(rng.standard_normal((B, Hq, D)) * 0.1)
    k = _bf(rng.standard_normal((B, Hkv, cap, D)))
    v = _bf(rng.standard_normal((B, Hkv, cap, D)))
    lo, hi = np.zeros(B, np.int32), np.full(B, n, np.int32)
    dense_ref, w = _reference(q, k, v, n, Hkv, 0.0)
    dense = orc.attn_decode_bf16(q, Hkv, cap, lo, hi, k, v, 1.0)
    np.testing.assert_allclose(dense, dense_ref, rtol=0, atol=1e-4 * np.abs(dense_ref).max())
    # tau = 0 keeps every weight
    np.testing.assert_array_equal(orc.attn_decode_bf16(q, Hkv, cap, lo, hi, k, v, 1.0, tau=0.0), dense)
    flat = np.sort(w.ravel())
    for target in (0.5 / n, 1.0 / n, 2.0 / n):
        i = int(np.clip(np.searchsorted(flat, target), 1, flat.size - 1))
        tau = float(0.5 * (flat[i - 1] + flat[i]))
        want, _ = _reference(q, k, v, n, Hkv, tau)
        got = orc.attn_decode_bf16(q, Hkv, cap, lo, hi, k, v, 1.0, tau=tau)
        kept = float((w >= tau).mean())
        assert 0.0 < kept < 1.0
        np.testing.assert_allclose(got, want, rtol=0, atol=1e-4 * np.abs(want).max())
        # the gate removes mass: the output moves away from the dense one
        assert np.abs(got - dense).max() > 1e-3 * np.abs(dense).max()
