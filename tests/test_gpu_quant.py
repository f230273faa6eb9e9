"""GPU parity: MLX-affine quantise / dequantise (bit-exact) and quantised
linear (fp32-accumulated GEMV, max-relative-error tolerance 1e-2)."""
import numpy as np
import pytest
import torch

from gpu_util import max_rel_err, to_np_bf16, to_np_u32

pytestmark = pytest.mark.gpu
TOL = 1e-2


@pytest.mark.parametrize("bits", [2, 3, 4, 5, 6, 8])
@pytest.mark.parametrize("src_bf16", [False, True])
def test_quantize_bit_exact(fm, orc, dev, bits, src_bf16):
    g = torch.Generator(device=dev).manual_seed(100 + bits)
    w = torch.randn(96, 2816, generator=g, device=dev) * 0.02
    if src_bf16:
        w = w.to(torch.bfloat16)
    wq, s, b = fm.quantize(w, bits)
    w_host = orc.bf16_to_f32(to_np_bf16(w)) if src_bf16 else w.cpu().numpy()
    owq, os_, ob = orc.quantize(w_host, bits)
    assert np.array_equal(to_np_u32(wq), owq)
    assert np.array_equal(to_np_bf16(s), os_) and np.array_equal(to_np_bf16(b), ob)


@pytest.mark.parametrize("bits", [4, 6, 8])
def test_dequantize_bit_exact(fm, orc, dev, bits):
    g = torch.Generator(device=dev).manual_seed(200 + bits)
    w = torch.randn(64, 704, generator=g, device=dev) * 0.02
    ql = fm.QuantizedLinear.from_float(w, bits)
    out = ql.dequantize()
    want = orc.dequantize(to_np_u32(ql.weight), to_np_bf16(ql.scales), to_np_bf16(ql.biases), 704, bits)
    assert np.array_equal(to_np_bf16(out), want)


def test_embed_rows_6bit(fm, orc, dev):
    g = torch.Generator(device=dev).manual_seed(7)
    w = torch.randn(1000, 2816, generator=g, device=dev) * 0.02
    ql = fm.QuantizedLinear.from_float(w, 6)
    ids = torch.tensor([0, 999, 17, 17, 500], device=dev)
    scale = 2816 ** 0.5
    out = ql.embed(ids, scale)
    deq = orc.dequantize(to_np_u32(ql.weight), to_np_bf16(ql.scales), to_np_bf16(ql.biases), 2816, 6)
    rs = orc.bf16_to_f32(orc.f32_to_bf16(np.float32([scale])))[0]
    want = orc.f32_to_bf16(orc.bf16_to_f32(deq[ids.cpu().numpy()]) * rs)
    assert np.array_equal(to_np_bf16(out), want)


@pytest.mark.parametrize("bits", [16, 4, 8])
@pytest.mark.parametrize("shape", [(128, 2816), (704, 2816), (2816, 704), (4096, 2816)])
@pytest.mark.parametrize("T", [1, 3, 17])
def test_qlinear_matches_oracle(fm, orc, dev, bits, shape, T):
    out_f, in_f = shape
    g = torch.Generator(device=dev).manual_seed(out_f + in_f + bits + T)
    w = torch.randn(out_f, in_f, generator=g, device=dev) * 0.02
    x = torch.randn(T, in_f, generator=g, device=dev).to(torch.bfloat16)
    ql = fm.QuantizedLinear.from_float(w, bits)
    y = ql.forward(x)
    xn = to_np_bf16(x)
    if bits == 16:
        want = orc.matmul_bf16(xn, to_np_bf16(ql.weight))
    else:
        want = orc.qmatmul(xn, to_np_u32(ql.weight), to_np_bf16(ql.scales), to_np_bf16(ql.biases), in_f, bits)
    assert max_rel_err(y.float().cpu().numpy(), want) <= TOL


def test_qlinear_rejects_bad_shapes(fm, dev):
    w = torch.randn(10, 128, device=dev)
    ql = fm.QuantizedLinear.from_float(w.to(torch.bfloat16), 16)
    with pytest.raises(fm.FmoeError) as ei:
        ql.forward(torch.zeros(1, 128, dtype=torch.bfloat16, device=dev))
    assert ei.value.code == -5


# The streaming tensor-core GEMV (T <= 8): decoder shapes, the 6-bit lm_head
# width, and K large enough to need column chunks accumulated in fp32.
@pytest.mark.parametrize("bits", [4, 6, 8])
@pytest.mark.parametrize("shape", [(4096, 2816), (2816, 4096), (2816, 8192), (2816, 2112), (272, 2816)])
@pytest.mark.parametrize("T", [1, 2, 8])
def test_qlinear_streaming_matches_oracle(fm, orc, dev, bits, shape, T):
    out_f, in_f = shape
    g = torch.Generator(device=dev).manual_seed(7 * out_f + in_f + bits + T)
    w = torch.randn(out_f, in_f, generator=g, device=dev) * 0.02
    x = torch.randn(T, in_f, generator=g, device=dev).to(torch.bfloat16)
    ql = fm.QuantizedLinear.from_float(w, bits)
    y = ql.forward(x)
    want = orc.qmatmul(to_np_bf16(x), to_np_u32(ql.weight), to_np_bf16(ql.scales), to_np_bf16(ql.biases), in_f,
                       bits)
    assert max_rel_err(y.float().cpu().numpy(), want) <= TOL
