"""fmoe_b200 — host-side mirror of flash-moe's quantised-MoE hot path over libfmoe.

Python binds the C ABI in include/fmoe.h through ctypes; torch supplies device
memory and streams only.  The classes mirror the reference's operator interface
for this path (names, argument meaning, error behaviour):

    QuantizedLinear.forward(x)          src/model/mlp.rs:14-26
    GeLUMLP.forward(x)                  src/model/mlp.rs:35-41
    Gemma4MoeBlock.forward(x)           src/model/moe.rs:315-470
    KVCache.update_and_fetch(k, v)      src/cache.rs:266-310   (see kv.py)
    Gemma4DecoderLayer.forward(x, ...)  src/model/mod.rs:67-119  (see model.py)
    Gemma4Model.decode_step()           src/model/mod.rs:135-363
    ExpertParallelMoeBlock.forward(x)   moe.rs:315-470 with experts split over GPUs (see ep.py)

There is no CPU fallback: every call goes to the CUDA kernels in
lib/libfmoe.so, and a missing library or device raises.
"""
from __future__ import annotations

import ctypes
import os

import torch

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "lib", "libfmoe.so")

FMOE_OK = 0
_ERRORS = {
    -1: "FMOE_ERR_INVALID",
    -2: "FMOE_ERR_ALIGN",
    -3: "FMOE_ERR_WORKSPACE",
    -4: "FMOE_ERR_CUDA",
    -5: "FMOE_ERR_UNSUPPORTED",
    -6: "FMOE_ERR_TIMEOUT",
    -7: "FMOE_ERR_NCCL",
    -8: "FMOE_ERR_ALLOC",
}


class FmoeError(RuntimeError):
    def __init__(self, code: int, msg: str):
        super().__init__(f"{_ERRORS.get(code, code)}: {msg}")
        self.code = code


class QWeightC(ctypes.Structure):
    _fields_ = [
        ("w", ctypes.c_void_p),
        ("scales", ctypes.c_void_p),
        ("biases", ctypes.c_void_p),
        ("out_features", ctypes.c_int32),
        ("in_features", ctypes.c_int32),
        ("bits", ctypes.c_int32),
        ("group_size", ctypes.c_int32),
        ("tiled", ctypes.c_void_p),
        ("tiled_kc", ctypes.c_int32),
        ("reserved", ctypes.c_int32),
    ]


class ExpertsC(ctypes.Structure):
    _fields_ = [
        ("base", ctypes.c_void_p),
        ("expert_stride", ctypes.c_int64),
        ("offsets", ctypes.c_int64 * 9),
        ("num_experts", ctypes.c_int32),
        ("first_expert", ctypes.c_int32),
        ("hidden", ctypes.c_int32),
        ("intermediate", ctypes.c_int32),
        ("bits", ctypes.c_int32),
        ("group_size", ctypes.c_int32),
        ("slot_of", ctypes.c_void_p),
    ]


class RouterC(ctypes.Structure):
    _fields_ = [
        ("proj", QWeightC),
        ("router_scale", ctypes.c_void_p),
        ("per_expert_scale", ctypes.c_void_p),
        ("logit_bias", ctypes.c_void_p),
        ("root_size", ctypes.c_float),
        ("eps", ctypes.c_float),
        ("use_norm", ctypes.c_int32),
        ("top_k", ctypes.c_int32),
    ]


class KvCacheC(ctypes.Structure):
    _fields_ = [
        ("mode", ctypes.c_int32),
        ("batch", ctypes.c_int32),
        ("kv_heads", ctypes.c_int32),
        ("head_dim", ctypes.c_int32),
        ("capacity", ctypes.c_int64),
        ("k_bits", ctypes.c_int32),
        ("v_bits", ctypes.c_int32),
        ("group_size", ctypes.c_int32),
        ("turbo_bits", ctypes.c_int32),
        ("k", ctypes.c_void_p),
        ("v", ctypes.c_void_p),
        ("k_scales", ctypes.c_void_p),
        ("k_biases", ctypes.c_void_p),
        ("v_scales", ctypes.c_void_p),
        ("v_biases", ctypes.c_void_p),
    ]


class KernelStatC(ctypes.Structure):
    _fields_ = [("name", ctypes.c_char * 64), ("launches", ctypes.c_int64), ("total_ms", ctypes.c_double)]


_P = ctypes.c_void_p
_I64 = ctypes.c_int64
_I = ctypes.c_int
_SZ = ctypes.c_size_t
_F = ctypes.c_float

# name -> (restype, argtypes); every symbol declared in include/fmoe.h.
SIGNATURES = {
    "fmoe_version": (_I, []),
    "fmoe_last_error": (_I, [ctypes.c_char_p, _SZ]),
    "fmoe_workspace_status": (_I, [_P, _I, _P]),
    "fmoe_wait_selftest": (_I, [_P, _SZ, _I, _P]),
    "fmoe_moe_block_forward_noalloc": (
        _I,
        [_P, _I64, ctypes.POINTER(RouterC), ctypes.POINTER(ExpertsC), _P, _P, _P, _P],
    ),
    "fmoe_moe_block_noalloc_status": (_I, [_I, _P]),
    "fmoe_profile_enable": (_I, [_I]),
    "fmoe_profile_read": (_I, [ctypes.POINTER(KernelStatC), _I, _I]),
    "fmoe_quantize": (_I, [_P, _I, _I64, _I64, _I, _I, _P, _P, _P, _P]),
    "fmoe_dequantize": (_I, [ctypes.POINTER(QWeightC), _P, _P]),
    "fmoe_embed_rows": (_I, [ctypes.POINTER(QWeightC), _P, _I64, _F, _P, _P]),
    "fmoe_qgemv_chunk": (ctypes.c_int32, [ctypes.c_int32, ctypes.c_int32, _I64, ctypes.c_int32]),
    "fmoe_qweight_tile_bytes": (_SZ, [ctypes.POINTER(QWeightC), ctypes.c_int32]),
    "fmoe_qweight_tile": (_I, [ctypes.POINTER(QWeightC), ctypes.c_int32, _P, _SZ, _P]),
    "fmoe_qlinear_workspace_bytes": (_SZ, [_I64, ctypes.POINTER(QWeightC)]),
    "fmoe_qlinear": (_I, [_P, _I64, ctypes.POINTER(QWeightC), _P, _P, _SZ, _P]),
    "fmoe_router_workspace_bytes": (_SZ, [_I64, ctypes.POINTER(RouterC)]),
    "fmoe_router": (_I, [_P, _I64, ctypes.POINTER(RouterC), _P, _P, _P, _P, _SZ, _P]),
    "fmoe_moe_workspace_bytes": (_SZ, [_I64, _I, ctypes.POINTER(ExpertsC)]),
    "fmoe_moe_experts": (_I, [_P, _I64, _I, _P, _P, ctypes.POINTER(ExpertsC), _P, _P, _SZ, _P]),
    "fmoe_moe_block_workspace_bytes": (_SZ, [_I64, ctypes.POINTER(RouterC), ctypes.POINTER(ExpertsC)]),
    "fmoe_moe_block_forward": (
        _I,
        [_P, _I64, ctypes.POINTER(RouterC), ctypes.POINTER(ExpertsC), _P, _P, _P, _P, _SZ, _P],
    ),
    "fmoe_kv_cache_bytes": (_SZ, [_I, _I, _I, _I, _I64]),
    "fmoe_kv_cache_init": (_I, [ctypes.POINTER(KvCacheC), _I, _I, _I, _I, _I64, _P, _SZ]),
    "fmoe_kv_append": (_I, [ctypes.POINTER(KvCacheC), _P, _P, _I64, _I64, _P, _I, _P]),
    "fmoe_attn_decode_workspace_bytes": (_SZ, [ctypes.POINTER(KvCacheC), _I]),
    "fmoe_attn_decode": (_I, [ctypes.POINTER(KvCacheC), _P, _I, _I64, _P, _F, _P, _P, _SZ, _P]),
    "fmoe_attn_decode_sparse_v": (_I, [ctypes.POINTER(KvCacheC), _P, _I, _I64, _F, _F, _P, _P]),
    "fmoe_turbo_round_trip": (_I, [_P, _I64, _I, _I, _P, _P]),
    "fmoe_decoder_workspace_bytes": (_SZ, [_I64, _P, ctypes.POINTER(KvCacheC)]),
    "fmoe_decoder_layer_forward": (_I, [_P, ctypes.POINTER(KvCacheC), _P, _I64, _I64, _P, _P, _SZ, _P]),
    "fmoe_decoder_layer_prefill_workspace_bytes": (_SZ, [_P, _I64]),
    "fmoe_decoder_layer_prefill": (_I, [_P, ctypes.POINTER(KvCacheC), _P, _I64, _I64, _I, _P, _P, _SZ, _P]),
    "fmoe_attn_prefill": (_I, [ctypes.POINTER(KvCacheC), _P, _I, _I64, _I64, _I, _P, _P, _P, _F, _P]),
    "fmoe_decoder_layer_prefill_ep_workspace_bytes": (_SZ, [_P, _I64, _I]),
    "fmoe_decoder_layer_prefill_ep": (_I, [_P, ctypes.POINTER(KvCacheC), _P, _P, _I64, _I64, _I, _P, _P, _SZ, _P]),
    "fmoe_mlp_workspace_bytes": (_SZ, [_I64, ctypes.POINTER(QWeightC)]),
    "fmoe_mlp_forward": (_I, [_P, _I64, ctypes.POINTER(QWeightC), ctypes.POINTER(QWeightC), ctypes.POINTER(QWeightC),
                              _P, _P, _SZ, _P]),
    "fmoe_lm_head_workspace_bytes": (_SZ, [_I64]),
    "fmoe_lm_head": (_I, [ctypes.POINTER(QWeightC), _P, _F, _P, _I64, _F, _P, _P, _P, _P, _SZ, _P]),
    "fmoe_sample_workspace_bytes": (_SZ, [_I64, _I64]),
    "fmoe_sample": (_I, [_P, _I64, _I64, _P, _I, _F, _F, _F, ctypes.c_uint64, _P, _I, _P, _P, _SZ, _P]),
    "fmoe_moe_prefill_prepare_bytes": (_SZ, [ctypes.POINTER(ExpertsC)]),
    "fmoe_moe_prefill_prepare": (_I, [ctypes.POINTER(ExpertsC), _P, _SZ, _P]),
    "fmoe_moe_prefill_workspace_bytes": (_SZ, [_I64, ctypes.POINTER(RouterC), ctypes.POINTER(ExpertsC)]),
    "fmoe_moe_prefill": (_I, [_P, _I64, ctypes.POINTER(RouterC), ctypes.POINTER(ExpertsC), _P, _P, _P, _P, _P, _SZ,
                              _P]),
    "fmoe_moe_prefill_experts_workspace_bytes": (_SZ, [_I64, _I, ctypes.POINTER(ExpertsC)]),
    "fmoe_moe_prefill_experts": (_I, [_P, _I64, _I, _P, _P, ctypes.POINTER(ExpertsC), _P, _P, _P, _SZ, _P]),
    "fmoe_ep_unique_id": (_I, [_P, _SZ]),
    "fmoe_ep_comm_init": (_I, [ctypes.POINTER(ctypes.c_void_p), _I, _I, _P, _SZ]),
    "fmoe_ep_comm_destroy": (_I, [_P]),
    "fmoe_ep_comm_abort": (_I, [_P]),
    "fmoe_ep_comm_status": (_I, [_P]),
    "fmoe_ep_p2p_init": (_I, [_P, _I64, _I, _I]),
    "fmoe_ep_moe_workspace_bytes": (_SZ, [_I, _I64, ctypes.POINTER(RouterC), ctypes.POINTER(ExpertsC)]),
    "fmoe_ep_moe_forward": (_I, [_P, _P, _I64, _I64, ctypes.POINTER(RouterC), ctypes.POINTER(ExpertsC), _P, _P, _P,
                                 _P, _I, _P, _SZ, _P]),
    "fmoe_decoder_ep_workspace_bytes": (_SZ, [_I64, _P, ctypes.POINTER(KvCacheC), _I, _I64]),
    "fmoe_decoder_layer_forward_ep": (_I, [_P, ctypes.POINTER(KvCacheC), _P, _I64, _P, _I, _P, _I64, _I64, _P, _P,
                                           _SZ, _P]),
    "fmoe_decode_step_workspace_bytes": (_SZ, [_P]),
    "fmoe_decode_step_prepare": (_I, [_P, _P, _SZ]),
    "fmoe_decode_step": (_I, [_P, _P, _P, _P, _P, _SZ, _P]),
}

_lib_handle = None


def lib() -> ctypes.CDLL:
    """Load libfmoe.so (raises if it has not been built)."""
    global _lib_handle
    if _lib_handle is None:
        if not os.path.exists(LIB_PATH):
            raise RuntimeError(f"libfmoe.so not built ({LIB_PATH}); run __graft_entry__.build()")
        h = ctypes.CDLL(LIB_PATH)
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(h, name)
            fn.restype = res
            fn.argtypes = args
        _lib_handle = h
    return _lib_handle


def last_error() -> str:
    buf = ctypes.create_string_buffer(512)
    lib().fmoe_last_error(buf, 512)
    return buf.value.decode()


def check(rc: int) -> None:
    if rc != FMOE_OK:
        raise FmoeError(rc, last_error())


def profile_enable(on: bool = True) -> None:
    """Bracket every library kernel launch with CUDA events (not during capture)."""
    check(lib().fmoe_profile_enable(int(on)))


def profile_read(reset: bool = True) -> dict:
    """{kernel name: (launches, total device ms)} since the last reset."""
    arr = (KernelStatC * 64)()
    n = lib().fmoe_profile_read(arr, 64, int(reset))
    if n < 0:
        check(n)
    return {arr[i].name.decode(): (arr[i].launches, arr[i].total_ms) for i in range(min(n, 64))}


def _ptr(t) -> int | None:
    return None if t is None else t.data_ptr()


def _stream(stream=None) -> int:
    if stream is None:
        stream = torch.cuda.current_stream()
    return stream.cuda_stream


def _need_cuda(*ts):
    for t in ts:
        if t is not None and not t.is_cuda:
            raise ValueError("fmoe: tensors must live on a CUDA device")


class _Workspace:
    """Grow-only device scratch buffer, zero-filled when (re)allocated: the
    router keeps completion counters in it that every call leaves at zero."""

    def __init__(self):
        self.buf = None

    def get(self, nbytes: int, device) -> torch.Tensor:
        if self.buf is None or self.buf.numel() < nbytes or self.buf.device != device:
            self.buf = torch.zeros(max(nbytes, 256), dtype=torch.uint8, device=device)
        return self.buf


# ---------------------------------------------------------------------------
# quantisation


def quantize(w: torch.Tensor, bits: int = 4, group_size: int = 64):
    """MLX-affine quantisation on the GPU -> (wq uint32, scales bf16, biases bf16)."""
    _need_cuda(w)
    rows, cols = w.shape
    w = w.contiguous()
    if w.dtype not in (torch.float32, torch.bfloat16):
        w = w.float()
    wq = torch.empty(rows, cols * bits // 32, dtype=torch.int32, device=w.device)
    s = torch.empty(rows, cols // group_size, dtype=torch.bfloat16, device=w.device)
    b = torch.empty_like(s)
    check(lib().fmoe_quantize(_ptr(w), int(w.dtype == torch.bfloat16), rows, cols, bits, group_size,
                              _ptr(wq), _ptr(s), _ptr(b), _stream()))
    return wq, s, b


def prefill_prep(experts, device):
    """Transposed scale / bias copy of an expert table for the prefill GEMMs
    (fmoe_moe_prefill_prepare; built once per table and kept on it)."""
    prep = getattr(experts, "_prefill_prep", None)
    if prep is None:
        e = experts.cstruct()
        nbytes = lib().fmoe_moe_prefill_prepare_bytes(ctypes.byref(e))
        if nbytes == 0:
            check(lib().fmoe_moe_prefill_prepare(ctypes.byref(e), None, 0, None))
        prep = torch.empty(nbytes, dtype=torch.uint8, device=device)
        check(lib().fmoe_moe_prefill_prepare(ctypes.byref(e), _ptr(prep), nbytes, _stream()))
        experts._prefill_prep = prep
    return prep


def mlp_forward(x: torch.Tensor, gate, up, down) -> torch.Tensor:
    """GeLUMLP::forward (src/model/mlp.rs:28-41) over T tokens on the tensor-core
    GEMM (fmoe_mlp_forward): x bf16 [T, hidden] -> bf16 [T, hidden]."""
    _need_cuda(x)
    x2 = x.reshape(-1, x.shape[-1]).to(torch.bfloat16).contiguous()
    T = x2.shape[0]
    g, u, d = gate.cstruct(), up.cstruct(), down.cstruct()
    ws = torch.empty(lib().fmoe_mlp_workspace_bytes(T, ctypes.byref(g)), dtype=torch.uint8, device=x.device)
    y = torch.empty(T, down.out_features, dtype=torch.bfloat16, device=x.device)
    check(lib().fmoe_mlp_forward(_ptr(x2), T, ctypes.byref(g), ctypes.byref(u), ctypes.byref(d), _ptr(y), _ptr(ws),
                                 ws.numel(), _stream()))
    return y.reshape(*x.shape[:-1], down.out_features)


class QuantizedLinear:
    """Mirror of QuantizedLinear (src/model/mlp.rs:4-26): packed uint32 weight,
    bf16 scales/biases; bits == 16 means a plain bf16 weight [out, in]."""

    def __init__(self, weight, scales=None, biases=None, bits=4, group_size=64, in_features=None):
        self.weight = weight
        self.scales = scales
        self.biases = biases
        self.bits = bits
        self.group_size = group_size
        self.out_features = weight.shape[0]
        self.in_features = in_features or (weight.shape[1] if bits == 16 else weight.shape[1] * 32 // bits)
        self.tiled, self.tiled_kc = None, 0
        self._ws = _Workspace()

    @classmethod
    def from_float(cls, w: torch.Tensor, bits=4, group_size=64):
        if bits == 16:
            return cls(w.to(torch.bfloat16).contiguous(), bits=16)
        wq, s, b = quantize(w, bits, group_size)
        return cls(wq, s, b, bits, group_size, in_features=w.shape[1])

    def cstruct(self) -> QWeightC:
        return QWeightC(_ptr(self.weight), _ptr(self.scales), _ptr(self.biases), self.out_features,
                        self.in_features, self.bits, self.group_size, _ptr(self.tiled), self.tiled_kc, 0)

    def tile(self, rows_total: int | None = None, accumulate: bool = False) -> "QuantizedLinear":
        """Add a copy of the weight in the decode GEMV's tile layout (one contiguous
        block per 16-row unit).  rows_total: the rows of every weight sharing this
        one's GEMV launch (they must be tiled alike); accumulate: that launch adds
        split-K slices (o_proj, dense MLP) rather than storing rows."""
        rows = self.out_features if rows_total is None else rows_total
        kc = lib().fmoe_qgemv_chunk(self.in_features, self.bits, rows, int(accumulate))
        if kc <= 0:
            raise FmoeError(-5, f"qweight {self.out_features}x{self.in_features} at {self.bits} bits: not tileable")
        self.tiled = None
        c = self.cstruct()
        nbytes = lib().fmoe_qweight_tile_bytes(ctypes.byref(c), kc)
        if nbytes == 0:
            raise FmoeError(-5, "qweight tile: unsupported shape")
        buf = torch.empty(nbytes, dtype=torch.uint8, device=self.weight.device)
        check(lib().fmoe_qweight_tile(ctypes.byref(c), kc, _ptr(buf), nbytes, _stream()))
        self.tiled, self.tiled_kc = buf, kc
        return self

    def dequantize(self) -> torch.Tensor:
        out = torch.empty(self.out_features, self.in_features, dtype=torch.bfloat16, device=self.weight.device)
        c = self.cstruct()
        check(lib().fmoe_dequantize(ctypes.byref(c), _ptr(out), _stream()))
        return out

    def embed(self, ids: torch.Tensor, scale: float = 1.0) -> torch.Tensor:
        """take + dequantize (+ x scale), src/model/mod.rs:145-160."""
        ids = ids.to(torch.int32).contiguous().view(-1)
        out = torch.empty(ids.numel(), self.in_features, dtype=torch.bfloat16, device=self.weight.device)
        c = self.cstruct()
        check(lib().fmoe_embed_rows(ctypes.byref(c), _ptr(ids), ids.numel(), scale, _ptr(out), _stream()))
        return out

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        _need_cuda(x)
        shape = x.shape
        x2 = x.reshape(-1, shape[-1]).contiguous()
        T = x2.shape[0]
        y = torch.empty(T, self.out_features, dtype=torch.bfloat16, device=x.device)
        c = self.cstruct()
        nbytes = lib().fmoe_qlinear_workspace_bytes(T, ctypes.byref(c))
        ws = self._ws.get(nbytes, x.device)
        check(lib().fmoe_qlinear(_ptr(x2), T, ctypes.byref(c), _ptr(y), _ptr(ws), ws.numel(), _stream()))
        return y.reshape(*shape[:-1], self.out_features)

    __call__ = forward


# ---------------------------------------------------------------------------
# experts (ECB layout)

ECB_TENSORS = ("gate.w", "gate.s", "gate.b", "up.w", "up.s", "up.b", "down.w", "down.s", "down.b")


def ecb_layout(hidden: int, inter: int, bits: int = 4, group: int = 64):
    """Byte sizes / offsets of the 9 per-expert tensors in ECB order
    (src/splitter.rs:405-457): returns (offsets, sizes, stride)."""
    wg = inter * hidden * bits // 8
    sg = inter * (hidden // group) * 2
    wd = hidden * inter * bits // 8
    sd = hidden * (inter // group) * 2
    sizes = [wg, sg, sg, wg, sg, sg, wd, sd, sd]
    offs = []
    o = 0
    for s in sizes:
        offs.append(o)
        o += s
    return offs, sizes, o


class ExpertTable:
    """All experts of one MoE layer resident in HBM in ECB expert-major order:
    one uint8 buffer [num_experts * stride] (expert e at e*stride)."""

    def __init__(self, buf: torch.Tensor, num_experts: int, hidden: int, inter: int, bits=4, group=64,
                 first_expert=0, slot_of: torch.Tensor | None = None):
        self.buf = buf
        self.slot_of = slot_of  # device int32 [num_experts]: expert e in slot slot_of[e] of buf (host tier)
        self.num_experts = num_experts
        self.hidden = hidden
        self.inter = inter
        self.bits = bits
        self.group = group
        self.first_expert = first_expert
        self.offsets, self.sizes, self.stride = ecb_layout(hidden, inter, bits, group)
        assert slot_of is not None or buf.numel() >= num_experts * self.stride

    @classmethod
    def random(cls, num_experts, hidden, inter, bits=4, group=64, std=0.02, seed=0, device="cuda"):
        """Synthetic experts: N(0, std) weights, MLX-affine quantised on the GPU
        (one quantise call per projection over all experts)."""
        offs, sizes, stride = ecb_layout(hidden, inter, bits, group)
        buf = torch.empty(num_experts * stride, dtype=torch.uint8, device=device)
        view = buf.view(num_experts, stride)
        gen = torch.Generator(device=device)
        gen.manual_seed(seed)
        for j, (o, i) in enumerate([(inter, hidden), (inter, hidden), (hidden, inter)]):
            w = torch.randn(num_experts * o, i, generator=gen, device=device, dtype=torch.float32) * std
            wq, s, b = quantize(w, bits, group)
            del w
            for t, src in enumerate((wq, s, b)):
                a = offs[3 * j + t]
                view[:, a:a + sizes[3 * j + t]].copy_(src.contiguous().view(torch.uint8).view(num_experts, -1))
        return cls(buf, num_experts, hidden, inter, bits, group)

    def tensor(self, e: int, name: str) -> torch.Tensor:
        j = ECB_TENSORS.index(name)
        off = e * self.stride + self.offsets[j]
        raw = self.buf[off:off + self.sizes[j]]
        rows = self.inter if j < 6 else self.hidden
        return raw.view(torch.int32 if j % 3 == 0 else torch.bfloat16).view(rows, -1)

    def cstruct(self) -> ExpertsC:
        return ExpertsC(_ptr(self.buf), self.stride, (ctypes.c_int64 * 9)(*self.offsets), self.num_experts,
                        self.first_expert, self.hidden, self.inter, self.bits, self.group, _ptr(self.slot_of))

    def to(self, device, non_blocking: bool = True) -> "ExpertTable":
        """The same table on another device (e.g. a pinned host copy -> HBM, asynchronously)."""
        return ExpertTable(self.buf.to(device, non_blocking=non_blocking), self.num_experts, self.hidden, self.inter,
                           self.bits, self.group, first_expert=self.first_expert,
                           slot_of=None if self.slot_of is None else self.slot_of.to(device))

    def shard(self, rank: int, world: int, copy: bool = False) -> "ExpertTable":
        """Experts [rank*E/world, (rank+1)*E/world) of this (whole) table, for
        expert parallelism: a view of the same bytes, or its own copy."""
        if self.first_expert != 0:
            raise ValueError("shard: not a whole table")
        from .ep import shard_range
        first, n = shard_range(self.num_experts, world, rank)
        buf = self.buf[first * self.stride:(first + n) * self.stride]
        return ExpertTable(buf.clone() if copy else buf, n, self.hidden, self.inter, self.bits, self.group,
                           first_expert=first)


def moe_experts(x: torch.Tensor, ids: torch.Tensor, weights: torch.Tensor, table: ExpertTable,
                ws: _Workspace | None = None) -> torch.Tensor:
    """Routed experts + weighted combine (src/model/moe.rs:361-466)."""
    _need_cuda(x, ids, weights)
    T, H = x.shape
    k = ids.shape[1]
    ids = ids.to(torch.int32).contiguous()
    weights = weights.to(torch.float32).contiguous()
    y = torch.empty(T, H, dtype=torch.bfloat16, device=x.device)
    c = table.cstruct()
    nbytes = lib().fmoe_moe_workspace_bytes(T, k, ctypes.byref(c))
    buf = (ws or _Workspace()).get(nbytes, x.device)
    check(lib().fmoe_moe_experts(_ptr(x.contiguous()), T, k, _ptr(ids), _ptr(weights), ctypes.byref(c), _ptr(y),
                                 _ptr(buf), buf.numel(), _stream()))
    return y


class Gemma4MoeBlock:
    """Mirror of Gemma4MoeBlock (src/model/moe.rs:298-312): router_proj,
    router_scale, per_expert_scale, root_size, rms_norm_eps, top_k, plus the
    layer's resident expert table.  `logit_bias` is the synthetic skew device of
    the prefill benchmark (absent in the reference; None disables it)."""

    def __init__(self, router_proj: QuantizedLinear, experts: ExpertTable, top_k=8, router_scale=None,
                 per_expert_scale=None, root_size=None, rms_norm_eps=1e-6, use_norm=False, logit_bias=None):
        self.router_proj = router_proj
        self.experts = experts
        self.top_k = top_k
        self.router_scale = router_scale
        self.per_expert_scale = per_expert_scale
        self.root_size = root_size if root_size is not None else experts.hidden ** -0.5
        self.rms_norm_eps = rms_norm_eps
        self.use_norm = use_norm
        self.logit_bias = logit_bias
        self._ws = _Workspace()

    def router_cstruct(self) -> RouterC:
        return RouterC(self.router_proj.cstruct(), _ptr(self.router_scale), _ptr(self.per_expert_scale),
                       _ptr(self.logit_bias), self.root_size, self.rms_norm_eps, int(self.use_norm), self.top_k)

    def route(self, x: torch.Tensor, want_logits=False):
        """Router only: (ids int32 [T,k], weights f32 [T,k], logits f32 [T,E] | None)."""
        x2 = x.reshape(-1, x.shape[-1]).contiguous()
        T = x2.shape[0]
        E = self.router_proj.out_features
        ids = torch.empty(T, self.top_k, dtype=torch.int32, device=x.device)
        w = torch.empty(T, self.top_k, dtype=torch.float32, device=x.device)
        lg = torch.empty(T, E, dtype=torch.float32, device=x.device) if want_logits else None
        r = self.router_cstruct()
        nbytes = lib().fmoe_router_workspace_bytes(T, ctypes.byref(r))
        buf = self._ws.get(nbytes, x.device)
        check(lib().fmoe_router(_ptr(x2), T, ctypes.byref(r), _ptr(ids), _ptr(w), _ptr(lg), _ptr(buf), buf.numel(),
                                _stream()))
        return ids, w, lg

    # Tokens above which forward() takes the tensor-core prefill path (the
    # decode GEMV path serves at most 128 tokens per call).
    PREFILL_MIN_TOKENS = 129

    def _prepared(self, device):
        return prefill_prep(self.experts, device)

    def forward_prefill(self, x: torch.Tensor, return_routing=False):
        """Router + experts over many tokens on the tcgen05 grouped-GEMM path
        (fmoe_moe_prefill): token-sorted expert tiles, fp32 accumulation."""
        _need_cuda(x)
        shape = x.shape
        x2 = x.reshape(-1, shape[-1]).contiguous()
        T = x2.shape[0]
        y = torch.empty_like(x2)
        ids = torch.empty(T, self.top_k, dtype=torch.int32, device=x.device)
        w = torch.empty(T, self.top_k, dtype=torch.float32, device=x.device)
        r = self.router_cstruct()
        e = self.experts.cstruct()
        prep = self._prepared(x.device)
        nbytes = lib().fmoe_moe_prefill_workspace_bytes(T, ctypes.byref(r), ctypes.byref(e))
        if nbytes == 0:
            check(lib().fmoe_moe_prefill(None, T, ctypes.byref(r), ctypes.byref(e), None, None, None, None, None, 0,
                                         None))
        buf = self._ws.get(nbytes, x.device)
        check(lib().fmoe_moe_prefill(_ptr(x2), T, ctypes.byref(r), ctypes.byref(e), _ptr(prep), _ptr(y), _ptr(ids),
                                     _ptr(w), _ptr(buf), buf.numel(), _stream()))
        y = y.reshape(shape)
        return (y, ids, w) if return_routing else y

    def forward(self, x: torch.Tensor, return_routing=False):
        _need_cuda(x)
        shape = x.shape
        x2 = x.reshape(-1, shape[-1]).contiguous()
        T = x2.shape[0]
        if T >= self.PREFILL_MIN_TOKENS:
            return self.forward_prefill(x, return_routing)
        y = torch.empty_like(x2)
        ids = torch.empty(T, self.top_k, dtype=torch.int32, device=x.device)
        w = torch.empty(T, self.top_k, dtype=torch.float32, device=x.device)
        r = self.router_cstruct()
        e = self.experts.cstruct()
        nbytes = lib().fmoe_moe_block_workspace_bytes(T, ctypes.byref(r), ctypes.byref(e))
        buf = self._ws.get(nbytes, x.device)
        check(lib().fmoe_moe_block_forward(_ptr(x2), T, ctypes.byref(r), ctypes.byref(e), _ptr(y), _ptr(ids), _ptr(w),
                                           _ptr(buf), buf.numel(), _stream()))
        y = y.reshape(shape)
        return (y, ids, w) if return_routing else y

    __call__ = forward


from .kv import KV_AFFINE, KV_BF16, KVCache, turbo_round_trip  # noqa: E402
from .model import GEMMA4_26B, Gemma4DecoderLayer, Gemma4Model  # noqa: E402
from .ep import (FMOE_EP_EXACT, FMOE_EP_FIXED, FMOE_EP_P2P, EPComm, ExpertParallelMoeBlock, PeerLost, PeerWatch,  # noqa: E402
                 shard_range)
from . import ecb  # noqa: E402
from .tier import HostExpertTier, TieredMoeBlock  # noqa: E402
from .sample import Sampler, sample_tokens  # noqa: E402
from . import safetensors  # noqa: E402
from . import split  # noqa: E402
