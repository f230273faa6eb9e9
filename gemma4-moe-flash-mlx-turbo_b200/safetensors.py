"""Resident checkpoint loader: safetensors files to HBM, quantised linears with
the reference's flexible naming and its load-time re-quantisation.

The reference loads MLX checkpoints (safetensors) through mlx-rs and builds
every QuantizedLinear with load_qlinear_flex (src/model/mod.rs:633-680): the
scales / biases are named `<prefix>.scales` / `.biases` (Qwen) or
`<prefix>.weight_scales` / `.weight_biases` (Gemma-4), and a bit width its
kernels lack (e.g. 5-bit) is dequantised and re-quantised at load time to the
largest supported width below it (4 when there is none).  Here the same, with
the supported widths being this library's decode kernels (4, 6, 8) and the
re-quantisation done on the GPU (fmoe_dequantize, then fmoe_quantize from the
bf16 weights, the order the reference uses: dequantize, then quantize).

Format (safetensors): u64 little-endian header length N, N bytes of JSON
{name: {"dtype", "shape", "data_offsets": [begin, end]}, "__metadata__": {...}},
then the data; offsets count from the end of the header.  Packed uint32
weights come back as int32 tensors (the same bits), bf16 as bfloat16.
"""
from __future__ import annotations

import json
import os
import struct

import numpy as np
import torch

_NP = {"U8": np.uint8, "I8": np.int8, "U16": np.uint16, "I16": np.int16, "F16": np.float16, "BF16": np.uint16,
       "U32": np.uint32, "I32": np.int32, "F32": np.float32, "U64": np.uint64, "I64": np.int64, "F64": np.float64,
       "BOOL": np.bool_}
_SIGNED = {"BF16": np.int16, "U16": np.int16, "U32": np.int32, "U64": np.int64}
QLINEAR_BITS = (4, 6, 8)        # widths the decode GEMV kernels serve (4 and 8 for every token count)
QLINEAR_GROUPS = (64,)          # the kernels' group size


class SafetensorsError(ValueError):
    pass


def read_header(path: str) -> tuple[dict, int]:
    """-> ({name: (dtype, shape, begin, end)}, absolute offset of the data)."""
    size = os.path.getsize(path)
    with open(path, "rb") as f:
        head = f.read(8)
        if len(head) < 8:
            raise SafetensorsError(f"{path}: shorter than the 8-byte header length")
        (n,) = struct.unpack("<Q", head)
        if n < 2 or 8 + n > size:
            raise SafetensorsError(f"{path}: header length {n} outside the file ({size} bytes)")
        try:
            hdr = json.loads(f.read(n))
        except (UnicodeDecodeError, json.JSONDecodeError) as e:
            raise SafetensorsError(f"{path}: header is not JSON ({e})") from None
    base = 8 + n
    out = {}
    for name, d in hdr.items():
        if name == "__metadata__":
            continue
        dt, shape, (b, e) = d["dtype"], tuple(d["shape"]), d["data_offsets"]
        if dt not in _NP:
            raise SafetensorsError(f"{path}: {name}: dtype {dt}")
        nbytes = int(np.prod(shape, dtype=np.int64)) * np.dtype(_NP[dt]).itemsize
        if not 0 <= b <= e or e - b != nbytes or base + e > size:
            raise SafetensorsError(f"{path}: {name}: data offsets [{b}, {e}) for {nbytes} bytes in a "
                                   f"{size - base}-byte data section")
        out[name] = (dt, shape, b, e)
    return out, base


def load(path: str, device="cuda", names=None) -> dict[str, torch.Tensor]:
    """Tensors of a safetensors file (all, or `names`) on `device`."""
    hdr, base = read_header(path)
    want = hdr.keys() if names is None else names
    out = {}
    with open(path, "rb") as f:
        for name in want:
            if name not in hdr:
                raise KeyError(f"{path}: no tensor {name}")
            dt, shape, b, e = hdr[name]
            f.seek(base + b)
            a = np.frombuffer(f.read(e - b), dtype=_NP[dt]).reshape(shape)
            t = torch.from_numpy(a.view(_SIGNED.get(dt, a.dtype)).copy())  # unsigned -> same-width signed bits
            out[name] = (t.view(torch.bfloat16) if dt == "BF16" else t).to(device)
    return out


def save(path: str, tensors: dict[str, np.ndarray | torch.Tensor], metadata: dict | None = None) -> None:
    """Write a safetensors file (numpy arrays, or torch tensors: bf16 kept as BF16,
    int32 packed weights written as U32)."""
    entries, blobs, off = {}, [], 0
    for name, t in tensors.items():
        if isinstance(t, torch.Tensor):
            t = t.detach().cpu()
            if t.dtype == torch.bfloat16:
                a, dt = t.view(torch.int16).numpy().view(np.uint16), "BF16"
            elif t.dtype == torch.int32:
                a, dt = t.numpy().view(np.uint32), "U32"
            else:
                a = t.numpy()
                dt = next(k for k, v in _NP.items() if np.dtype(v) == a.dtype and k != "BF16")
        else:
            a = np.asarray(t)
            dt = next(k for k, v in _NP.items() if np.dtype(v) == a.dtype and k != "BF16")
        raw = np.ascontiguousarray(a).tobytes()
        entries[name] = {"dtype": dt, "shape": list(a.shape), "data_offsets": [off, off + len(raw)]}
        blobs.append(raw)
        off += len(raw)
    if metadata:
        entries["__metadata__"] = metadata
    head = json.dumps(entries).encode()
    head += b" " * (-len(head) % 8)
    with open(path, "wb") as f:
        f.write(struct.pack("<Q", len(head)))
        f.write(head)
        for raw in blobs:
            f.write(raw)


def read_raw(path: str, names=None) -> dict[str, tuple[str, tuple, bytes]]:
    """{name: (dtype, shape, raw bytes)} of a safetensors file (all, or `names`)."""
    hdr, base = read_header(path)
    out = {}
    with open(path, "rb") as f:
        for name in (hdr.keys() if names is None else names):
            dt, shape, b, e = hdr[name]
            f.seek(base + b)
            out[name] = (dt, shape, f.read(e - b))
    return out


def save_raw(path: str, tensors: dict[str, tuple[str, tuple, bytes]], metadata: dict | None = None) -> None:
    """Write {name: (dtype, shape, raw bytes)} as a safetensors file."""
    entries, off = {}, 0
    for name, (dt, shape, raw) in tensors.items():
        if len(raw) != int(np.prod(shape, dtype=np.int64)) * np.dtype(_NP[dt]).itemsize:
            raise SafetensorsError(f"{name}: {len(raw)} bytes for {dt} {tuple(shape)}")
        entries[name] = {"dtype": dt, "shape": list(shape), "data_offsets": [off, off + len(raw)]}
        off += len(raw)
    if metadata:
        entries["__metadata__"] = metadata
    head = json.dumps(entries).encode()
    head += b" " * (-len(head) % 8)
    with open(path, "wb") as f:
        f.write(struct.pack("<Q", len(head)))
        f.write(head)
        for _, _, raw in tensors.values():
            f.write(raw)


def nearest_supported_bits(bits: int, supported=QLINEAR_BITS) -> int:
    """The largest supported width <= bits, else 4 (src/model/mod.rs:637-643)."""
    below = [b for b in supported if b <= bits]
    return max(below) if below else 4


def load_qlinear(weights: dict, prefix: str, bits: int, group_size: int = 64, supported=QLINEAR_BITS,
                 groups=QLINEAR_GROUPS):
    """load_qlinear_flex (src/model/mod.rs:648-680): the QuantizedLinear at
    `prefix` from a loaded tensor dict; a width outside `supported` is
    re-quantised on the GPU to nearest_supported_bits(bits), and a group size
    outside `groups` to group 64 (the kernels' one group size).  A bf16 weight
    with no scales is kept as a plain bf16 linear (bits 16), the form the
    library's router takes."""
    from . import QuantizedLinear, quantize

    w = weights.get(f"{prefix}.weight")
    if w is None:
        raise KeyError(f"missing weight: {prefix}.weight")
    s = weights.get(f"{prefix}.scales", weights.get(f"{prefix}.weight_scales"))
    if s is None and w.dtype == torch.bfloat16:
        return QuantizedLinear(w, bits=16)
    if s is None:
        raise KeyError(f"missing scales for: {prefix}")
    b = weights.get(f"{prefix}.biases", weights.get(f"{prefix}.weight_biases"))
    if b is None:
        raise KeyError(f"missing biases for: {prefix}")
    cols = w.shape[1] * 32 // bits
    if (w.shape[0] != s.shape[0] or s.shape != b.shape or cols * bits != w.shape[1] * 32
            or cols != s.shape[1] * group_size):
        raise ValueError(f"{prefix}: weight {tuple(w.shape)}, scales {tuple(s.shape)}, biases {tuple(b.shape)} "
                         f"are not a {bits}-bit, group-{group_size} quantised linear")
    q = QuantizedLinear(w, s, b, bits, group_size, in_features=cols)
    if bits in supported and group_size in groups:
        return q
    target = bits if bits in supported else nearest_supported_bits(bits, supported)
    tg = group_size if group_size in groups else 64
    wq, s2, b2 = quantize(q.dequantize(), target, tg)  # bf16 weights, as the reference's dequantize gives
    return QuantizedLinear(wq, s2, b2, target, tg, in_features=cols)
