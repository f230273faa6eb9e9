"""ECB ("expert-centric binary") files: one MoE layer's routed experts, expert-major.

The reference's splitter writes one ECB file per layer (src/splitter.rs:405-457) and its
expert manager parses the header and reads expert e's tensors at
header_size + e * per_expert_stride + tensor offset (src/memory.rs:323-377, 571-607).
Format (little-endian):

    header (header_size bytes, 16384 as written): b"ECB1", u32 num_experts,
        u32 per_expert_stride, u32 num_tensors, u32 header_size, then per tensor
        u32 per-expert byte stride, u32 dtype code, u32 ndim, ndim x u32 per-expert shape
    data: for every expert, its tensors back to back in header order

dtype codes: 0 uint8, 1 uint32, 2 bfloat16, 3 float16, 4 float32, 5 int32.  For
Gemma-4 the nine tensors are gate.w gate.s gate.b up.w up.s up.b down.w down.s down.b
(src/splitter.rs:566-577) — the order ExpertTable and fmoe_experts_t use.

Here the data section goes to HBM once per layer (every expert resident): the whole
table, or one rank's contiguous slice for expert parallelism.
"""
from __future__ import annotations

import os
import struct

import numpy as np
import torch

MAGIC = b"ECB1"
HEADER_SIZE = 16384
DTYPE_CODES = {0: np.uint8, 1: np.uint32, 2: np.uint16, 3: np.float16, 4: np.float32, 5: np.int32}
_CODE_OF = {"w": 1, "s": 2, "b": 2}


class EcbError(ValueError):
    pass


def read_header(path: str) -> dict:
    """Parse an ECB header -> {num_experts, stride, header_size, tensors: [(stride, code, shape), ...]}."""
    with open(path, "rb") as f:
        fixed = f.read(20)
        if len(fixed) < 20 or fixed[:4] != MAGIC:
            raise EcbError(f"{path}: not an ECB file (bad magic)")
        num_experts, stride, num_tensors, header_size = struct.unpack("<4I", fixed[4:20])
        if header_size < 20:
            raise EcbError(f"{path}: header size {header_size}")
        desc = f.read(header_size - 20)
    tensors, pos = [], 0
    for _ in range(num_tensors):
        if pos + 12 > len(desc):
            raise EcbError(f"{path}: truncated tensor descriptors")
        tstride, code, ndim = struct.unpack_from("<3I", desc, pos)
        pos += 12
        shape = struct.unpack_from(f"<{ndim}I", desc, pos)
        pos += 4 * ndim
        if code not in DTYPE_CODES:
            raise EcbError(f"{path}: dtype code {code}")
        tensors.append((tstride, code, tuple(shape)))
    if sum(t[0] for t in tensors) != stride:
        raise EcbError(f"{path}: tensor strides sum to {sum(t[0] for t in tensors)}, header says {stride}")
    size = os.path.getsize(path)
    if size < header_size + num_experts * stride:
        raise EcbError(f"{path}: {size} bytes, expected {header_size + num_experts * stride}")
    return {"num_experts": num_experts, "stride": stride, "header_size": header_size, "tensors": tensors}


def layer_shape(hdr: dict) -> dict:
    """hidden / intermediate / bits / group of a Gemma-4 expert layer from its nine
    tensor descriptors (gate.w [I, H*bits/32] uint32, gate.s [I, H/group] bf16, ...)."""
    t = hdr["tensors"]
    if len(t) != 9:
        raise EcbError(f"expected 9 expert tensors, found {len(t)}")
    codes = [c for _, c, _ in t]
    if codes != [1, 2, 2] * 3:
        raise EcbError(f"dtype codes {codes}: expected uint32 weights with bf16 scales / biases")
    (gw, gs, gb, uw, us, ub, dw, ds, db) = [s for _, _, s in t]
    inter, hidden = gs[0], dw[0]
    group = hidden // gs[1]
    bits = gw[1] * 32 // hidden
    if (gw[0], uw, us, ub, gb) != (inter, gw, gs, gs, gs) or ds != (hidden, inter // group) or db != ds \
            or dw != (hidden, inter * bits // 32) or hidden % group or bits not in (2, 3, 4, 5, 6, 8):
        raise EcbError("tensor shapes are not a gate / up / down expert triple")
    return {"hidden": hidden, "inter": inter, "bits": bits, "group": group}


def load(path: str, device="cuda", experts: tuple[int, int] | None = None, pin: bool = False):
    """ECB file -> ExpertTable in HBM.  experts = (first, count) keeps only that
    contiguous slice (one rank's share for expert parallelism); only its bytes are
    read.  pin=True returns the host copy in pinned memory instead (the optional
    host tier; ExpertTable.to(device) moves it)."""
    from . import ExpertTable, ecb_layout

    hdr = read_header(path)
    shp = layer_shape(hdr)
    E, stride = hdr["num_experts"], hdr["stride"]
    first, n = (0, E) if experts is None else experts
    if first < 0 or n < 1 or first + n > E:
        raise EcbError(f"experts [{first}, {first + n}) outside [0, {E})")
    offs, sizes, lstride = ecb_layout(shp["hidden"], shp["inter"], shp["bits"], shp["group"])
    if lstride != stride or [s for s, _, _ in hdr["tensors"]] != sizes:
        raise EcbError("tensor strides differ from the MLX-affine layout of these shapes")
    host = torch.empty(n * stride, dtype=torch.uint8, pin_memory=pin)
    with open(path, "rb") as f:
        f.seek(hdr["header_size"] + first * stride)
        nread = f.readinto(memoryview(host.numpy()))
    if nread != n * stride:
        raise EcbError(f"{path}: short read")
    buf = host if pin else host.to(device)
    return ExpertTable(buf, n, shp["hidden"], shp["inter"], shp["bits"], shp["group"], first_expert=first)


CODE_OF_DTYPE = {"U8": 0, "U32": 1, "BF16": 2, "F16": 3, "F32": 4, "I32": 5}


def write_tensors(path: str, tensors) -> None:
    """ECB file from expert-stacked tensors: tensors = [(dtype name, per-expert
    shape, uint8 array [E, per-expert bytes]), ...] in file order (the
    splitter's write_ecb_file, src/splitter.rs:405-457): header, then for every
    expert its slice of each tensor back to back."""
    E = tensors[0][2].shape[0]
    if any(t[2].shape[0] != E for t in tensors):
        raise EcbError("write_tensors: tensors disagree on the expert count")
    stride = sum(t[2].shape[1] for t in tensors)
    hdr = bytearray(HEADER_SIZE)
    struct.pack_into("<4s4I", hdr, 0, MAGIC, E, stride, len(tensors), HEADER_SIZE)
    pos = 20
    for dt, shape, data in tensors:
        if pos + 12 + 4 * len(shape) > HEADER_SIZE:
            raise EcbError("write_tensors: descriptors exceed the header")
        struct.pack_into(f"<3I{len(shape)}I", hdr, pos, data.shape[1], CODE_OF_DTYPE[dt], len(shape), *shape)
        pos += 12 + 4 * len(shape)
    with open(path, "wb") as f:
        f.write(bytes(hdr))
        f.write(np.ascontiguousarray(np.concatenate([t[2] for t in tensors], axis=1)).tobytes())


def write(path: str, table) -> None:
    """ExpertTable (whole layer) -> ECB file in the splitter's format."""
    if table.first_expert != 0:
        raise EcbError("write: not a whole table")
    H, I, bits, g = table.hidden, table.inter, table.bits, table.group
    shapes = [(I, H * bits // 32), (I, H // g), (I, H // g)] * 2 + [(H, I * bits // 32), (H, I // g), (H, I // g)]
    hdr = bytearray(HEADER_SIZE)
    struct.pack_into("<4s4I", hdr, 0, MAGIC, table.num_experts, table.stride, 9, HEADER_SIZE)
    pos = 20
    for size, shape, kind in zip(table.sizes, shapes, ["w", "s", "b"] * 3):
        struct.pack_into(f"<3I{len(shape)}I", hdr, pos, size, _CODE_OF[kind], len(shape), *shape)
        pos += 12 + 4 * len(shape)
    data = table.buf[: table.num_experts * table.stride].cpu().numpy()
    with open(path, "wb") as f:
        f.write(bytes(hdr))
        f.write(data.tobytes())
