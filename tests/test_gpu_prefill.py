"""GPU parity: the prefill MoE block (fmoe_moe_prefill: tcgen05 grouped GEMMs
over token-sorted expert tiles) against the CPU oracle's router + expert loop
(src/model/moe.rs:315-470), and against the decode path where both run.

Routing as in the decode tests (ids equal where the k-th / (k+1)-th logit gap
exceeds 1e-3).  Outputs: max |gpu - oracle| / max |oracle| <= 1e-2, evaluated
on the GPU's own routing; the prefill path rounds each expert's output to
bf16 before the weighted combine, as the reference's quantized_matmul output
is, which stays well inside that bound.
"""
import numpy as np
import pytest
import torch

from gpu_util import max_rel_err, to_np_bf16
from test_gpu_moe import E, H, I, K, _check_routing, _oracle_experts

pytestmark = pytest.mark.gpu
TOL = 1e-2


@pytest.fixture(scope="module")
def layer(fm, dev):
    table = fm.ExpertTable.random(E, H, I, seed=2002, device=dev)
    g = torch.Generator(device=dev).manual_seed(2002)
    wr = (torch.randn(E, H, generator=g, device=dev) * 0.02).to(torch.bfloat16)
    bias = torch.randn(E, generator=g, device=dev)  # Zipf-like skew of BASELINE config 2
    return table, wr, bias, table.buf.cpu().numpy()


@pytest.mark.parametrize("T,skew", [(64, False), (200, True), (512, True), (131, False)])
def test_prefill_matches_oracle(fm, orc, dev, layer, T, skew):
    table, wr, bias, host = layer
    g = torch.Generator(device=dev).manual_seed(3000 + T)
    x = torch.randn(T, H, generator=g, device=dev).to(torch.bfloat16)
    block = fm.Gemma4MoeBlock(fm.QuantizedLinear(wr, bits=16), table, top_k=K, logit_bias=bias if skew else None)
    y, ids, w = block.forward_prefill(x, return_routing=True)
    torch.cuda.synchronize()
    kw = {"logit_bias": bias.cpu().numpy()} if skew else {}
    _check_routing(orc, x, wr, ids, w, K, **kw)
    want = _oracle_experts(orc, table, host, x, ids, w)
    err = max_rel_err(y.float().cpu().numpy(), want)
    assert err <= TOL, err
    y2 = block.forward_prefill(x)  # deterministic
    assert torch.equal(y, y2)


def test_prefill_matches_decode_path(fm, dev, layer):
    table, wr, _, _ = layer
    T = 96
    g = torch.Generator(device=dev).manual_seed(4)
    x = torch.randn(T, H, generator=g, device=dev).to(torch.bfloat16)
    block = fm.Gemma4MoeBlock(fm.QuantizedLinear(wr, bits=16), table, top_k=K)
    y_dec, ids_dec, _ = block.forward(x, return_routing=True)  # T <= 128: the GEMV path
    y_pf, ids_pf, _ = block.forward_prefill(x, return_routing=True)
    assert torch.equal(ids_dec, ids_pf)
    assert max_rel_err(y_pf.float().cpu().numpy(), y_dec.float().cpu().numpy()) <= TOL


def test_prefill_one_hot_expert_many_tiles(fm, orc, dev, layer):
    """A huge bias on 8 experts routes every token to them: 300 tokens per
    expert = three 128-row tiles each, the last one partial."""
    table, wr, _, host = layer
    T = 300
    bias = torch.zeros(E, device=dev)
    hot = torch.tensor([3, 17, 40, 41, 77, 100, 126, 127], device=dev)
    bias[hot] = 1e4
    g = torch.Generator(device=dev).manual_seed(5)
    x = torch.randn(T, H, generator=g, device=dev).to(torch.bfloat16)
    block = fm.Gemma4MoeBlock(fm.QuantizedLinear(wr, bits=16), table, top_k=K, logit_bias=bias)
    y, ids, w = block.forward_prefill(x, return_routing=True)
    assert set(np.unique(ids.cpu().numpy()).tolist()) == set(hot.cpu().numpy().tolist())
    want = _oracle_experts(orc, table, host, x, ids, w)
    assert max_rel_err(y.float().cpu().numpy(), want) <= TOL


def test_prefill_many_pairs_equals_halves(fm, dev, layer):
    """T = 1000 (8000 pairs: the routing lists are built by many CTAs) gives
    bit-identically the rows of two T = 500 calls (one-CTA lists): every
    token's routing and expert arithmetic is independent of its batch."""
    table, wr, bias, _ = layer
    T = 1000
    g = torch.Generator(device=dev).manual_seed(8)
    x = torch.randn(T, H, generator=g, device=dev).to(torch.bfloat16)
    block = fm.Gemma4MoeBlock(fm.QuantizedLinear(wr, bits=16), table, top_k=K, logit_bias=bias)
    y, ids, _ = block.forward_prefill(x, return_routing=True)
    y0, ids0, _ = block.forward_prefill(x[:500], return_routing=True)
    y1, ids1, _ = block.forward_prefill(x[500:], return_routing=True)
    assert torch.equal(ids, torch.cat([ids0, ids1]))
    assert torch.equal(y, torch.cat([y0, y1]))


def test_forward_dispatches_prefill_above_128_tokens(fm, dev, layer):
    table, wr, _, _ = layer
    T = 160
    g = torch.Generator(device=dev).manual_seed(6)
    x = torch.randn(T, H, generator=g, device=dev).to(torch.bfloat16)
    block = fm.Gemma4MoeBlock(fm.QuantizedLinear(wr, bits=16), table, top_k=K)
    assert torch.equal(block.forward(x), block.forward_prefill(x))
