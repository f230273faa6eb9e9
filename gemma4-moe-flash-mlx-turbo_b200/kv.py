"""KV cache and decode attention over libfmoe (host-side mirror of src/cache.rs).

KVCache mirrors the reference's per-layer cache (src/cache.rs:161-310):

    KVCache.new() / new_with_window(w)                 plain bf16 storage
    KVCache.new_quantized(head_dim, bits[, window])     bf16 storage behind the
                                                        TurboQuant round trip
    KVCache.new_affine(head_dim[, window])              WHT-rotated affine K4/V8
                                                        (the benchmark's quantised
                                                        KV; no reference counterpart)
    offset() / stored_len() / update_and_fetch(k, v)

The reference concatenates new rows onto growing arrays and keeps the last
`window` positions; here the cache is a ring preallocated in HBM (capacity =
window, or max_positions for full attention), appends write slot
p % capacity, and decode attention reads the ring in place.  So
update_and_fetch returns the cache itself (the "fetched" K/V), which
`attend(q, scale)` consumes — the SDPA of src/model/gemma4_attention.rs:95-104.
"""
from __future__ import annotations

import ctypes

import torch

from . import FMOE_OK, KvCacheC, _need_cuda, _ptr, _stream, check, lib

KV_BF16 = 0
KV_AFFINE = 1


class KVCache:
    """One attention layer's KV cache for `batch` sequences that advance together."""

    def __init__(self, batch: int, kv_heads: int, head_dim: int, max_positions: int, window: int | None = None,
                 mode: int = KV_BF16, turbo_bits: int = 0, device=None):
        if turbo_bits and mode != KV_BF16:
            raise ValueError("turbo_bits applies to the bf16 storage mode")
        self.batch, self.kv_heads, self.head_dim = batch, kv_heads, head_dim
        self.window = window
        self.mode = mode
        self.turbo_bits = turbo_bits
        cap = window if window is not None else max_positions
        self.capacity = (cap + 15) // 16 * 16 if window is None else cap
        nbytes = lib().fmoe_kv_cache_bytes(mode, batch, kv_heads, head_dim, self.capacity)
        if nbytes == 0:
            raise ValueError(f"unsupported KV cache shape: batch={batch} kv_heads={kv_heads} head_dim={head_dim} "
                             f"capacity={self.capacity} (head_dim 256/512, capacity a multiple of 16)")
        device = torch.device("cuda") if device is None else torch.device(device)
        self.buf = torch.empty(nbytes, dtype=torch.uint8, device=device)
        self.c = KvCacheC()
        check(lib().fmoe_kv_cache_init(ctypes.byref(self.c), mode, batch, kv_heads, head_dim, self.capacity,
                                       _ptr(self.buf), nbytes))
        self.c.turbo_bits = turbo_bits  # the decoder layer's append applies it too
        self._offset = 0
        self._ws = None
        self._ws_heads = 0

    # constructors named after the reference's (src/cache.rs:184-223)
    @classmethod
    def new(cls, batch, kv_heads, head_dim, max_positions, device=None):
        return cls(batch, kv_heads, head_dim, max_positions, None, KV_BF16, 0, device)

    @classmethod
    def new_with_window(cls, batch, kv_heads, head_dim, window, device=None):
        return cls(batch, kv_heads, head_dim, window, window, KV_BF16, 0, device)

    @classmethod
    def new_quantized(cls, batch, kv_heads, head_dim, bits, max_positions, window=None, device=None):
        return cls(batch, kv_heads, head_dim, max_positions, window, KV_BF16, bits, device)

    @classmethod
    def new_affine(cls, batch, kv_heads, head_dim, max_positions, window=None, device=None):
        return cls(batch, kv_heads, head_dim, max_positions, window, KV_AFFINE, 0, device)

    def offset(self) -> int:
        """Monotonic position count (the RoPE offset), src/cache.rs:226-228."""
        return self._offset

    def stored_len(self) -> int:
        """Positions held (attendable), src/cache.rs:232-239."""
        return min(self._offset, self.capacity)

    def batch_view(self, b0: int, nb: int) -> "KVCache":
        """Sequences [b0, b0 + nb) of this cache as a cache of batch nb over the
        same storage (a decoder layer call takes at most 8 sequences; larger
        batches run as several calls on views of one cache)."""
        if b0 < 0 or nb < 1 or b0 + nb > self.batch:
            raise ValueError(f"batch_view: [{b0}, {b0 + nb}) outside batch {self.batch}")
        v = object.__new__(KVCache)
        v.__dict__.update(self.__dict__)
        v.batch = nb
        v._ws = None
        v._ws_heads = 0
        c = KvCacheC()
        ctypes.pointer(c)[0] = self.c
        c.batch = nb
        rows = b0 * self.kv_heads * self.capacity  # rows of the sequences before b0
        D = self.head_dim
        if self.mode == KV_BF16:
            row_bytes = {"k": 2 * D, "v": 2 * D}
        else:
            row_bytes = {"k": D // 2, "v": D, "k_scales": D // 32, "k_biases": D // 32, "v_scales": D // 32,
                         "v_biases": D // 32}
        for name, rb in row_bytes.items():
            p = getattr(self.c, name)
            if p:
                setattr(c, name, p + rows * rb)
        v.c = c
        return v

    # -- views of the stored arrays (tests and debugging) -------------------
    def _view(self, ptr, dtype, inner):
        off = ptr - self.buf.data_ptr()
        esz = torch.tensor([], dtype=dtype).element_size()
        n = self.batch * self.kv_heads * self.capacity * inner
        return self.buf[off:off + n * esz].view(dtype).view(self.batch, self.kv_heads, self.capacity, inner)

    def arrays(self) -> dict:
        D = self.head_dim
        if self.mode == KV_BF16:
            return {"k": self._view(self.c.k, torch.bfloat16, D), "v": self._view(self.c.v, torch.bfloat16, D)}
        return {
            "k": self._view(self.c.k, torch.int32, D // 8),
            "k_scales": self._view(self.c.k_scales, torch.bfloat16, D // 64),
            "k_biases": self._view(self.c.k_biases, torch.bfloat16, D // 64),
            "v": self._view(self.c.v, torch.int32, D // 4),
            "v_scales": self._view(self.c.v_scales, torch.bfloat16, D // 64),
            "v_biases": self._view(self.c.v_biases, torch.bfloat16, D // 64),
        }

    def slot(self, pos: int) -> int:
        return pos % self.capacity

    # -- the reference's interface ------------------------------------------
    def update(self, keys: torch.Tensor, values: torch.Tensor, pos_dev: torch.Tensor | None = None) -> None:
        """Append keys/values bf16 [batch, kv_heads, T_new, head_dim] at offset()."""
        _need_cuda(keys, values)
        B, H, T, D = keys.shape
        if (B, H, D) != (self.batch, self.kv_heads, self.head_dim) or values.shape != keys.shape:
            raise ValueError(f"kv append: got {tuple(keys.shape)} / {tuple(values.shape)}, cache is "
                             f"[{self.batch}, {self.kv_heads}, T, {self.head_dim}]")
        k = keys.to(torch.bfloat16).contiguous()
        v = values.to(torch.bfloat16).contiguous()
        check(lib().fmoe_kv_append(ctypes.byref(self.c), _ptr(k), _ptr(v), T, self._offset, _ptr(pos_dev),
                                   self.turbo_bits, _stream()))
        self._offset += T

    def update_and_fetch(self, keys: torch.Tensor, values: torch.Tensor) -> "KVCache":
        """KVCache::update_and_fetch (src/cache.rs:266-310): append, then hand
        back what attention reads — the cache itself, read in place."""
        self.update(keys, values)
        return self

    def attend_sparse_v(self, q: torch.Tensor, tau: float, scale: float = 1.0,
                        n_valid: int | None = None) -> torch.Tensor:
        """Sparse-V decode attention (fmoe_attn_decode_sparse_v; the reference's
        sparse_v_attention, src/model/gemma4_attention.rs:196-234): softmax
        weights below tau set to zero, not renormalised.  q bf16 [batch,
        q_heads, head_dim] -> bf16 [batch, q_heads, head_dim]."""
        _need_cuda(q)
        B, Hq, D = q.shape
        if B != self.batch or D != self.head_dim:
            raise ValueError(f"attend_sparse_v: q {tuple(q.shape)} vs cache batch {self.batch}, head_dim {D}")
        out = torch.empty(B, Hq, D, dtype=torch.bfloat16, device=q.device)
        n = self.stored_len() if n_valid is None else n_valid
        qc = q.to(torch.bfloat16).contiguous()
        check(lib().fmoe_attn_decode_sparse_v(ctypes.byref(self.c), _ptr(qc), Hq, n, scale, tau, _ptr(out),
                                              _stream()))
        return out

    def attend_prefill(self, q: torch.Tensor, k_new: torch.Tensor, v_new: torch.Tensor, pos0: int,
                       window: int | None = None, scale: float = 1.0) -> torch.Tensor:
        """Prefill SDPA (fmoe_attn_prefill) of T new tokens of this one-sequence
        cache: q bf16 [T, q_heads, head_dim], k_new / v_new bf16 [kv_heads, T,
        head_dim] (the new rows as they will be stored); positions < pos0 come
        from the ring.  window: the cache's own by default.  Returns bf16 [T,
        q_heads, head_dim]; the cache is not modified."""
        _need_cuda(q, k_new, v_new)
        T, Hq, D = q.shape
        if self.batch != 1 or D != self.head_dim or tuple(k_new.shape) != (self.kv_heads, T, D) or \
                v_new.shape != k_new.shape:
            raise ValueError(f"attend_prefill: q {tuple(q.shape)}, k_new {tuple(k_new.shape)} vs cache batch "
                             f"{self.batch}, kv_heads {self.kv_heads}, head_dim {self.head_dim}")
        win = self.window if window is None else window
        out = torch.empty(T, Hq, D, dtype=torch.bfloat16, device=q.device)
        qc, kc, vc = (t.to(torch.bfloat16).contiguous() for t in (q, k_new, v_new))
        check(lib().fmoe_attn_prefill(ctypes.byref(self.c), _ptr(qc), Hq, T, pos0, win or 0, _ptr(kc), _ptr(vc),
                                      _ptr(out), scale, _stream()))
        return out

    def workspace_bytes(self, q_heads: int) -> int:
        return lib().fmoe_attn_decode_workspace_bytes(ctypes.byref(self.c), q_heads)

    def attend(self, q: torch.Tensor, scale: float = 1.0, n_valid: int | None = None,
               n_valid_dev: torch.Tensor | None = None) -> torch.Tensor:
        """Decode SDPA of q bf16 [batch, q_heads, head_dim] (one token per
        sequence) over the stored positions -> bf16 [batch, q_heads, head_dim]."""
        _need_cuda(q)
        B, Hq, D = q.shape
        if B != self.batch or D != self.head_dim:
            raise ValueError(f"attend: q {tuple(q.shape)} vs cache batch {self.batch}, head_dim {self.head_dim}")
        nbytes = self.workspace_bytes(Hq)
        if nbytes == 0:
            raise ValueError(f"attend: unsupported q_heads {Hq} for {self.kv_heads} kv heads")
        if self._ws is None or self._ws.numel() < nbytes or self._ws.device != q.device:
            self._ws = torch.zeros(nbytes, dtype=torch.uint8, device=q.device)  # merge counters start at zero
        out = torch.empty_like(q, dtype=torch.bfloat16)
        n = self.stored_len() if n_valid is None else n_valid
        qc = q.to(torch.bfloat16).contiguous()
        check(lib().fmoe_attn_decode(ctypes.byref(self.c), _ptr(qc), Hq, n, _ptr(n_valid_dev), scale, _ptr(out),
                                     _ptr(self._ws), self._ws.numel(), _stream()))
        return out

    def status(self) -> int:
        """Synchronise and read the attention workspace's status word."""
        if self._ws is None:
            return FMOE_OK
        return lib().fmoe_workspace_status(_ptr(self._ws), 1, _stream())


def turbo_round_trip(x: torch.Tensor, bits: int) -> torch.Tensor:
    """TurboQuant quantise -> dequantise of bf16 rows [..., head_dim]
    (turbo_round_trip_kv, src/cache.rs:94-129)."""
    _need_cuda(x)
    D = x.shape[-1]
    xc = x.to(torch.bfloat16).contiguous()
    out = torch.empty_like(xc)
    check(lib().fmoe_turbo_round_trip(_ptr(xc), xc.numel() // D, D, bits, _ptr(out), _stream()))
    return out
