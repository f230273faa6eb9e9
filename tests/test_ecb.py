"""ECB files (src/splitter.rs:405-457 writes them, src/memory.rs:323-377 parses the
header): write -> parse -> load round trip on the golden expert table, slices for
expert parallelism, and rejection of malformed headers.  CPU only."""
import os
import struct

import numpy as np
import pytest
import torch

GOLD = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


@pytest.fixture()
def table(fm):
    d = np.load(os.path.join(GOLD, "moe_small.npz"))
    H, I, E = (int(v) for v in d["dims"][:3])
    t = fm.ExpertTable(torch.from_numpy(d["buf"].copy()), E, H, I)
    assert t.offsets == [int(o) for o in d["offsets"]] and t.stride == int(d["stride"])
    return t


def test_ecb_round_trip_and_header(fm, table, tmp_path):
    p = str(tmp_path / "layer0.ecb")
    fm.ecb.write(p, table)
    hdr = fm.ecb.read_header(p)
    assert hdr["num_experts"] == table.num_experts and hdr["stride"] == table.stride
    assert hdr["header_size"] == 16384 and len(hdr["tensors"]) == 9
    assert [t[0] for t in hdr["tensors"]] == table.sizes
    assert fm.ecb.layer_shape(hdr) == {"hidden": table.hidden, "inter": table.inter, "bits": 4, "group": 64}
    assert os.path.getsize(p) == 16384 + table.num_experts * table.stride
    back = fm.ecb.load(p, device="cpu")
    assert torch.equal(back.buf, table.buf) and back.first_expert == 0
    # expert e's gate.s at header + e * stride + offset (memory.rs:571-607)
    raw = open(p, "rb").read()
    e = 5
    o = 16384 + e * table.stride + table.offsets[1]
    assert raw[o:o + table.sizes[1]] == table.tensor(e, "gate.s").view(torch.int16).numpy().tobytes()


@pytest.mark.parametrize("rank,world", [(0, 2), (1, 2), (3, 4)])
def test_ecb_slice_for_expert_parallelism(fm, table, tmp_path, rank, world):
    p = str(tmp_path / "layer.ecb")
    fm.ecb.write(p, table)
    first, n = fm.shard_range(table.num_experts, world, rank)
    part = fm.ecb.load(p, device="cpu", experts=(first, n))
    want = table.shard(rank, world)
    assert part.first_expert == want.first_expert == first and part.num_experts == n
    assert torch.equal(part.buf, want.buf)


def test_ecb_pinned_host_copy(fm, table, tmp_path):
    if not torch.cuda.is_available():
        pytest.skip("pinned host memory needs a CUDA driver")
    p = str(tmp_path / "layer.ecb")
    fm.ecb.write(p, table)
    host = fm.ecb.load(p, pin=True)
    assert host.buf.is_pinned()


def test_ecb_rejects_bad_files(fm, table, tmp_path):
    p = str(tmp_path / "bad.ecb")
    fm.ecb.write(p, table)
    raw = bytearray(open(p, "rb").read())
    for mutate, msg in [(lambda b: b.__setitem__(slice(0, 4), b"XXXX"), "magic"),
                        (lambda b: struct.pack_into("<I", b, 8, table.stride + 16), "strides"),
                        (lambda b: b.__delitem__(slice(len(b) - 100, len(b))), "bytes")]:
        bad = bytearray(raw)
        mutate(bad)
        open(p, "wb").write(bytes(bad))
        with pytest.raises(fm.ecb.EcbError, match=msg):
            fm.ecb.load(p, device="cpu")
    with pytest.raises(fm.ecb.EcbError):
        fm.ecb.write(p, table)
        fm.ecb.load(p, device="cpu", experts=(6, 4))
