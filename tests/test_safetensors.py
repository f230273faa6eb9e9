"""CPU checks of the safetensors loader (safetensors.py): write / read round
trip, header validation, the flexible scale / bias naming of the reference's
load_qlinear_flex (src/model/mod.rs:648-680) and its bit-width fallback."""
import struct

import numpy as np
import pytest
import torch


@pytest.fixture(scope="module")
def st(fm):
    return fm.safetensors


def test_round_trip(st, tmp_path):
    g = np.random.default_rng(0)
    tensors = {
        "a.weight": torch.from_numpy(g.integers(-2**31, 2**31, (4, 10), dtype=np.int64).astype(np.int32)),
        "a.scales": torch.randn(4, 5).to(torch.bfloat16),
        "f32": g.standard_normal((3, 2)).astype(np.float32),
        "u8": np.arange(7, dtype=np.uint8),
    }
    path = str(tmp_path / "m.safetensors")
    st.save(path, tensors, metadata={"format": "mlx"})
    hdr, base = st.read_header(path)
    assert hdr["a.weight"][0] == "U32" and hdr["a.scales"][0] == "BF16" and base % 8 == 0
    got = st.load(path, device="cpu")
    assert torch.equal(got["a.weight"], tensors["a.weight"])
    assert got["a.scales"].dtype == torch.bfloat16 and torch.equal(got["a.scales"], tensors["a.scales"])
    assert np.array_equal(got["f32"].numpy(), tensors["f32"]) and np.array_equal(got["u8"].numpy(), tensors["u8"])
    only = st.load(path, device="cpu", names=["u8"])
    assert list(only) == ["u8"]
    with pytest.raises(KeyError):
        st.load(path, device="cpu", names=["nope"])


def test_header_validation(st, tmp_path):
    p = tmp_path / "bad.safetensors"
    p.write_bytes(b"\x01\x02")
    with pytest.raises(st.SafetensorsError):
        st.read_header(str(p))
    p.write_bytes(struct.pack("<Q", 1000) + b"{}")
    with pytest.raises(st.SafetensorsError):
        st.read_header(str(p))
    head = b'{"x": {"dtype": "F32", "shape": [4], "data_offsets": [0, 12]}}'
    p.write_bytes(struct.pack("<Q", len(head)) + head + bytes(16))  # 4 floats need 16 bytes
    with pytest.raises(st.SafetensorsError):
        st.read_header(str(p))
    head = b'{"x": {"dtype": "F32", "shape": [4], "data_offsets": [0, 16]}}'
    p.write_bytes(struct.pack("<Q", len(head)) + head + bytes(8))  # data section too short
    with pytest.raises(st.SafetensorsError):
        st.read_header(str(p))


def test_nearest_supported_bits(st):
    assert [st.nearest_supported_bits(b) for b in (2, 3, 4, 5, 6, 7, 8)] == [4, 4, 4, 4, 6, 6, 8]
    ref = (2, 3, 4, 6, 8)  # the reference's own list gives 5 -> 4, 7 -> 6
    assert [st.nearest_supported_bits(b, ref) for b in (2, 5, 7)] == [2, 4, 6]


@pytest.mark.parametrize("names", [(".scales", ".biases"), (".weight_scales", ".weight_biases")])
def test_load_qlinear_flex_naming(st, names):
    w = torch.zeros(8, 128 * 4 // 32, dtype=torch.int32)
    s = torch.ones(8, 2, dtype=torch.bfloat16)
    weights = {"m.weight": w, "m" + names[0]: s, "m" + names[1]: s * 0}
    q = st.load_qlinear(weights, "m", 4)
    assert (q.out_features, q.in_features, q.bits) == (8, 128, 4) and q.scales is s
    with pytest.raises(KeyError, match="missing biases"):
        st.load_qlinear({"m.weight": w, "m.scales": s}, "m", 4)
    with pytest.raises(ValueError):
        st.load_qlinear(weights, "m", 8)  # shapes are not an 8-bit layout
