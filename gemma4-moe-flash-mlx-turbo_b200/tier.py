"""Optional pinned-host tier for the routed experts.

The reference keeps experts on SSD, pages them in through mmap and hides the latency
with prefetchers (src/memory.rs: ExpertMemoryManager, reactive group prefetch
:644-736, zero-copy extraction :571-607).  Here every expert normally lives in HBM;
when HBM is short, this tier keeps each layer's expert table in pinned host memory and
a per-layer HBM cache of `slots` expert slots.  Before a layer's routed experts run,
the experts its router picked that are not cached are copied host -> HBM with
cudaMemcpyAsync on a copy stream (least recently used slot first), the layer's device
slot map (fmoe_experts_t.slot_of) is updated, and the compute stream waits on the
copies' event.  Like the reference (moe.rs:355-359) this needs the routed ids on the
host, so a tiered block is not capturable in a CUDA graph.
"""
from __future__ import annotations

import numpy as np
import torch

from . import ExpertTable, Gemma4MoeBlock, QuantizedLinear, moe_experts


def plan_slots(need, slot_of: np.ndarray, owner: np.ndarray, used: np.ndarray, clock: int) -> list[tuple[int, int]]:
    """Slot bookkeeping of one ensure() call (host only): every needed expert
    already in a slot is marked used at `clock`; each missing one gets a free
    slot, else the least recently used slot whose expert is not needed now.
    slot_of (expert -> slot, -1 on the host only), owner (slot -> expert, -1
    free) and used (slot -> last clock) are updated in place.  Returns the
    (expert, slot) copies to issue, in order."""
    for e in need:
        if slot_of[e] >= 0:
            used[slot_of[e]] = clock
    copies = []
    for e in [int(e) for e in need if slot_of[e] < 0]:
        free = np.flatnonzero(owner < 0)
        if free.size:
            s = int(free[0])
        else:
            cand = np.flatnonzero(used < clock)
            s = int(cand[np.argmin(used[cand])])
            slot_of[owner[s]] = -1
        owner[s] = e
        slot_of[e] = s
        used[s] = clock
        copies.append((e, s))
    return copies


class HostExpertTier:
    """host_tables: one whole-layer ExpertTable per layer in pinned host memory (e.g.
    ecb.load(..., pin=True)); slots: HBM expert slots per layer (>= the distinct
    experts one call can route to, i.e. min(T * top_k, E))."""

    def __init__(self, host_tables: list[ExpertTable], slots: int, device="cuda"):
        if not host_tables:
            raise ValueError("HostExpertTier: no layers")
        self.device = torch.device(device)
        self.host = host_tables
        self.slots = slots
        self.copy_stream = torch.cuda.Stream(device=self.device)
        self.layers = []
        for t in host_tables:
            if t.first_expert != 0 or not t.buf.is_pinned():
                raise ValueError("HostExpertTier: whole-layer tables in pinned host memory expected")
            if slots < 1 or slots > t.num_experts:
                raise ValueError(f"HostExpertTier: {slots} slots for {t.num_experts} experts")
            hbm = torch.empty(slots * t.stride, dtype=torch.uint8, device=self.device)
            slot_of = torch.zeros(t.num_experts, dtype=torch.int32, device=self.device)
            self.layers.append({
                "hbm": hbm,
                "slot_of_dev": slot_of,
                "slot_of": np.full(t.num_experts, -1, np.int64),   # expert -> slot (-1: on the host only)
                "owner": np.full(slots, -1, np.int64),             # slot -> expert
                "used": np.zeros(slots, np.int64),                 # last use (LRU clock)
                "staging": torch.zeros(t.num_experts, dtype=torch.int32).pin_memory(),
                "table": ExpertTable(hbm, t.num_experts, t.hidden, t.inter, t.bits, t.group, slot_of=slot_of),
            })
        self.clock = 0
        self.hits = self.misses = self.bytes_copied = 0

    def table(self, layer: int) -> ExpertTable:
        """The layer's HBM view (slot map included) for the expert kernels."""
        return self.layers[layer]["table"]

    def ensure(self, layer: int, ids: torch.Tensor, stream=None) -> None:
        """Make every expert in `ids` resident in the layer's slots; the current (or
        given) stream waits for the copies."""
        L, host = self.layers[layer], self.host[layer]
        stream = torch.cuda.current_stream(self.device) if stream is None else stream
        need = np.unique(ids.detach().cpu().numpy().astype(np.int64))  # the host sync of moe.rs:355-359
        need = need[(need >= 0) & (need < host.num_experts)]
        if need.size > self.slots:
            raise ValueError(f"layer {layer}: {need.size} routed experts exceed {self.slots} slots")
        self.clock += 1
        copies = plan_slots(need, L["slot_of"], L["owner"], L["used"], self.clock)
        self.hits += need.size - len(copies)
        self.misses += len(copies)
        if not copies:
            return
        self.copy_stream.wait_stream(stream)  # slots may still be read by earlier calls on `stream`
        with torch.cuda.stream(self.copy_stream):
            st = host.stride
            for e, s in copies:
                L["hbm"][s * st:(s + 1) * st].copy_(host.buf[e * st:(e + 1) * st], non_blocking=True)
                self.bytes_copied += st
            L["staging"].copy_(torch.from_numpy(np.maximum(L["slot_of"], 0).astype(np.int32)))
            L["slot_of_dev"].copy_(L["staging"], non_blocking=True)
        stream.wait_stream(self.copy_stream)


class TieredMoeBlock(Gemma4MoeBlock):
    """Gemma4MoeBlock whose experts come through a HostExpertTier (decode sizes)."""

    def __init__(self, router_proj: QuantizedLinear, tier: HostExpertTier, layer: int, **kw):
        super().__init__(router_proj, tier.table(layer), **kw)
        self.tier, self.layer = tier, layer

    def forward(self, x: torch.Tensor, return_routing=False):
        shape = x.shape
        x2 = x.reshape(-1, shape[-1]).contiguous()
        ids, w, _ = self.route(x2)
        self.tier.ensure(self.layer, ids)
        y = moe_experts(x2, ids, w, self.tier.table(self.layer), self._ws).reshape(shape)
        return (y, ids, w) if return_routing else y

    __call__ = forward
