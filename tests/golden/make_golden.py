"""Generates the small fixtures in tests/golden/ (run from the repo root).

  lcg_signs_seed42.npy  first 512 signs of deterministic_signs(n, 42)
                        (src/cache.rs:29-43), computed here in pure Python with
                        exact 64-bit arithmetic, independent of the C oracle.
  lloyd_max.json        the N(0,1) Lloyd-Max tables of src/cache.rs:67-89.
  quant_small.npz       seeded fp32 [8, 256] and its 2/4/6/8-bit MLX-affine
                        quantisation + dequantisation by the oracle.
  moe_small.npz         a seeded MoE block (H=128, I=64, E=8, k=2, T=3) with the
                        oracle's routing and output.
  turbo_small.npz       seeded bf16 [6, 256] rows and the oracle's TurboQuant
                        3-bit round trip.
  sample_small.npz      seeded fp32 logits [4, 512], recent-token lists (empty
                        slots, duplicates, out-of-range ids) and the sampling
                        oracle's tokens for a grid of (temperature, top_p,
                        penalty) at call numbers 0..2, plus its first uniforms.
"""
import json
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(os.path.dirname(HERE)))
import oracle  # noqa: E402


def lcg_signs(n, seed):
    state = seed
    out = []
    for _ in range(n):
        state = (state * 6364136223846793005 + 1442695040888963407) % (1 << 64)
        out.append(1.0 if (state >> 63) & 1 == 0 else -1.0)
    return np.array(out, np.float32)


LLOYD = {
    "2": {"centroids": [-1.510, -0.453, 0.453, 1.510], "boundaries": [-0.982, 0.0, 0.982]},
    "3": {"centroids": [-2.152, -1.344, -0.756, -0.245, 0.245, 0.756, 1.344, 2.152],
          "boundaries": [-1.748, -1.050, -0.501, 0.0, 0.501, 1.050, 1.748]},
    "4": {"centroids": [-2.733, -2.069, -1.618, -1.256, -0.942, -0.657, -0.388, -0.128,
                        0.128, 0.388, 0.657, 0.942, 1.256, 1.618, 2.069, 2.733],
          "boundaries": [-2.401, -1.844, -1.437, -1.099, -0.800, -0.522, -0.258, 0.0,
                         0.258, 0.522, 0.800, 1.099, 1.437, 1.844, 2.401]},
}


def ecb_layout(hidden, inter, bits=4, group=64):
    wg = inter * hidden * bits // 8
    sg = inter * (hidden // group) * 2
    wd = hidden * inter * bits // 8
    sd = hidden * (inter // group) * 2
    sizes = [wg, sg, sg, wg, sg, sg, wd, sd, sd]
    offs = list(np.cumsum([0] + sizes[:-1]))
    return [int(o) for o in offs], sizes, int(sum(sizes))


def main():
    rng = np.random.default_rng(20260101)
    np.save(os.path.join(HERE, "lcg_signs_seed42.npy"), lcg_signs(512, 42))
    with open(os.path.join(HERE, "lloyd_max.json"), "w") as f:
        json.dump(LLOYD, f, indent=1)

    w = (rng.standard_normal((8, 256)) * 0.02).astype(np.float32)
    q = {"w": w}
    for bits in (2, 4, 6, 8):
        wq, s, b = oracle.quantize(w, bits)
        q[f"wq{bits}"], q[f"s{bits}"], q[f"b{bits}"] = wq, s, b
        q[f"deq{bits}"] = oracle.dequantize(wq, s, b, 256, bits)
    np.savez_compressed(os.path.join(HERE, "quant_small.npz"), **q)

    H, I, E, K, T = 128, 64, 8, 2, 3
    x = oracle.f32_to_bf16(rng.standard_normal((T, H)).astype(np.float32))
    wr = oracle.f32_to_bf16((rng.standard_normal((E, H)) * 0.02).astype(np.float32))
    offs, sizes, stride = ecb_layout(H, I)
    buf = np.zeros(E * stride, np.uint8)
    for e in range(E):
        for j, (o, i) in enumerate([(I, H), (I, H), (H, I)]):
            wq, s, b = oracle.quantize((rng.standard_normal((o, i)) * 0.02).astype(np.float32), 4)
            for t, arr in enumerate((wq, s, b)):
                off = e * stride + offs[3 * j + t]
                buf[off:off + sizes[3 * j + t]] = arr.view(np.uint8).ravel()
    ids, wts, lg = oracle.router(x, wr, K)
    y32, y16 = oracle.moe_experts(x, ids, wts, buf, stride, offs, H, I)
    np.savez_compressed(os.path.join(HERE, "moe_small.npz"), x=x, wr=wr, buf=buf, stride=stride,
                        offsets=np.array(offs, np.int64), ids=ids, weights=wts, logits=lg, y32=y32, y16=y16,
                        dims=np.array([H, I, E, K, T]))

    v = oracle.f32_to_bf16(rng.standard_normal((6, 256)).astype(np.float32))
    out, idx, nrm = oracle.turbo_round_trip(v, 3)
    np.savez_compressed(os.path.join(HERE, "turbo_small.npz"), v=v, out=out, idx=idx, norm=nrm)

    sample_fixture()


SAMPLE_CASES = [(0.0, 1.0, 1.0), (0.0, 1.0, 1.3), (0.7, 1.0, 1.0), (0.7, 0.9, 1.15), (1.5, 0.5, 1.0)]


def sample_fixture():
    from oracle import sample as osmp

    rng = np.random.default_rng(7)
    lg = (rng.standard_normal((4, 512)) * 2.0).astype(np.float32)
    recent = rng.integers(-1, 520, size=(4, 16)).astype(np.int32)
    recent[:, 1] = recent[:, 0]
    toks = np.array([[osmp.sample(lg, recent, T, p, pen, seed=99, step=s) for s in range(3)]
                     for T, p, pen in SAMPLE_CASES], np.int32)
    np.savez_compressed(os.path.join(HERE, "sample_small.npz"), logits=lg, recent=recent,
                        cases=np.array(SAMPLE_CASES, np.float32), tokens=toks,
                        uniforms=osmp.uniforms(99, 0, 0, 8))


if __name__ == "__main__":
    main()
