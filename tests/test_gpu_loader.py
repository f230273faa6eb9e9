"""GPU checks of the resident loader's re-quantisation (safetensors.load_qlinear,
the reference's load_qlinear_flex, src/model/mod.rs:648-680): a 5-bit linear
read from a safetensors file becomes the 4-bit linear that the oracle gets by
dequantising (bf16) and quantising again — bit-exact — and its products stay
within the linear tolerance (max |a - b| / max |b| <= 1e-2) of the oracle's
product with that 4-bit weight; widths the kernels serve load unchanged."""
import numpy as np
import pytest
import torch

from gpu_util import max_rel_err, to_np_bf16

pytestmark = pytest.mark.gpu


def _bf(a_u16):
    return torch.from_numpy(np.ascontiguousarray(a_u16).view(np.int16)).view(torch.bfloat16)


def test_five_bit_linear_requantised_to_four(fm, orc, dev, tmp_path):
    g = np.random.default_rng(5)
    rows, cols = 96, 2816
    w = (g.standard_normal((rows, cols)) * 0.05).astype(np.float32)
    wq5, s5, b5 = orc.quantize(w, 5)
    path = str(tmp_path / "m.safetensors")
    fm.safetensors.save(path, {"layer.weight": wq5, "layer.weight_scales": _bf(s5), "layer.weight_biases": _bf(b5),
                               "dense.weight": orc.quantize(w, 8)[0], "dense.scales": _bf(orc.quantize(w, 8)[1]),
                               "dense.biases": _bf(orc.quantize(w, 8)[2])})
    weights = fm.safetensors.load(path, device=dev)
    q = fm.safetensors.load_qlinear(weights, "layer", 5)
    assert (q.bits, q.in_features, q.out_features) == (4, cols, rows)
    d = orc.dequantize(wq5, s5, b5, cols, 5)  # bf16 bits
    wq4, s4, b4 = orc.quantize(orc.bf16_to_f32(d), 4)
    assert np.array_equal(q.weight.cpu().numpy().view(np.uint32), wq4)
    assert np.array_equal(to_np_bf16(q.scales), s4) and np.array_equal(to_np_bf16(q.biases), b4)
    x = torch.randn(3, cols, device=dev).to(torch.bfloat16)
    y = q(x)
    want = orc.qmatmul(to_np_bf16(x), wq4, s4, b4, cols, 4)
    assert max_rel_err(y.float().cpu().numpy(), want) <= 1e-2
    q8 = fm.safetensors.load_qlinear(weights, "dense", 8)  # served as is
    assert q8.bits == 8 and q8.weight.data_ptr() == weights["dense.weight"].data_ptr()
