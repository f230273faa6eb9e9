"""GPU: the optional pinned-host expert tier (fmoe_experts_t.slot_of).  A layer
whose experts live in pinned host memory and reach HBM through a cache of 32
slots gives bit-identical outputs to the resident table, across calls that
evict and refill slots; the prefill path refuses slot-mapped tables."""
import pytest
import torch

pytestmark = pytest.mark.gpu
H, I, E, K = 2816, 704, 128, 8


def test_tiered_block_equals_resident(fm, dev):
    table = fm.ExpertTable.random(E, H, I, seed=61, device=dev)
    host = fm.ExpertTable(table.buf.cpu().pin_memory(), E, H, I)
    g = torch.Generator(device=dev).manual_seed(62)
    wr = (torch.randn(E, H, generator=g, device=dev) * 0.02).to(torch.bfloat16)
    router = fm.QuantizedLinear(wr, bits=16)
    resident = fm.Gemma4MoeBlock(router, table, top_k=K)
    tier = fm.HostExpertTier([host], slots=32, device=dev)
    tiered = fm.TieredMoeBlock(router, tier, 0, top_k=K)
    xs = [torch.randn(4, H, generator=g, device=dev).to(torch.bfloat16) for _ in range(5)]
    for x in xs + xs[:2]:  # the repeats hit slots still cached or refill evicted ones
        y0, i0, w0 = resident.forward(x, return_routing=True)
        y1, i1, w1 = tiered.forward(x, return_routing=True)
        torch.cuda.synchronize()
        assert torch.equal(i0, i1) and torch.equal(w0, w1)
        assert torch.equal(y0, y1)
    assert tier.misses > 32  # more distinct experts than slots: evictions happened
    assert tier.bytes_copied == tier.misses * table.stride
    with pytest.raises(fm.FmoeError, match="slot map"):
        fm.Gemma4MoeBlock(router, tier.table(0), top_k=K).forward_prefill(torch.randn(200, H, device=dev).to(
            torch.bfloat16))
