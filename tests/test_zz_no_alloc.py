"""fmoe_moe_block_forward_noalloc — the MoE block entry point for callers that
cannot allocate device memory when they run the layer (an engine whose memory
pool owns the whole device budget, a plugin host that forbids library
allocations, a decode loop that cannot afford cudaMalloc's synchronisation).
It runs on the library's own static scratch array instead of a caller
workspace.  It launches the same kernels on the same inputs as
fmoe_moe_block_forward, so its outputs must be bit-identical to that entry
point's, call after call, and its device status word must stay OK.

Named test_zz_* so pytest collects it last.
"""
import ctypes

import pytest
import torch

pytestmark = pytest.mark.gpu


def _noalloc(fm, block, x):
    T = x.shape[0]
    y = torch.empty_like(x)
    ids = torch.empty(T, block.top_k, dtype=torch.int32, device=x.device)
    w = torch.empty(T, block.top_k, dtype=torch.float32, device=x.device)
    r = block.router_cstruct()
    e = block.experts.cstruct()
    rc = fm.lib().fmoe_moe_block_forward_noalloc(x.data_ptr(), T, ctypes.byref(r), ctypes.byref(e), y.data_ptr(),
                                                 ids.data_ptr(), w.data_ptr(),
                                                 torch.cuda.current_stream().cuda_stream)
    fm.check(rc)
    return y, ids, w


def _status(fm):
    return fm.lib().fmoe_moe_block_noalloc_status(0, torch.cuda.current_stream().cuda_stream)


@pytest.mark.parametrize("H,I,E,K,T", [(256, 128, 16, 4, 3), (2816, 704, 128, 8, 1), (2816, 704, 128, 8, 16)])
def test_noalloc_matches_workspace_entry_point(fm, dev, H, I, E, K, T):
    table = fm.ExpertTable.random(E, H, I, seed=H + E, device=dev)
    g = torch.Generator(device=dev).manual_seed(H + T)
    wr = (torch.randn(E, H, generator=g, device=dev) * 0.02).to(torch.bfloat16)
    block = fm.Gemma4MoeBlock(fm.QuantizedLinear(wr, bits=16), table, top_k=K)
    for call in range(2):  # two calls in a row share (and must clear) the static scratch
        x = torch.randn(T, H, generator=g, device=dev).to(torch.bfloat16)
        y_ref, ids_ref, w_ref = block.forward(x, return_routing=True)
        y, ids, w = _noalloc(fm, block, x)
        torch.cuda.synchronize()
        assert _status(fm) == 0, call
        assert torch.equal(ids, ids_ref), call
        assert torch.equal(w, w_ref), call
        assert torch.equal(y, y_ref), call  # same kernels, same inputs: bit-identical


def test_noalloc_rejects_oversize(fm, dev):
    H, I, E, K, T = 2816, 704, 128, 8, 128
    table = fm.ExpertTable.random(E, H, I, seed=5, device=dev)
    wr = torch.zeros(E, H, dtype=torch.bfloat16, device=dev)
    block = fm.Gemma4MoeBlock(fm.QuantizedLinear(wr, bits=16), table, top_k=K)
    x = torch.zeros(T, H, dtype=torch.bfloat16, device=dev)
    with pytest.raises(fm.FmoeError) as ei:
        _noalloc(fm, block, x)
    assert ei.value.code == -3 and "static" in str(ei.value)
