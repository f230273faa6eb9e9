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
