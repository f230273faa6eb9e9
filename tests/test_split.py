"""CPU checks of the split-checkpoint loader (split.py, the reference's
load_gemma4_model, src/model/mod.rs:405-617): a two-layer synthetic split
directory (config.json with per-component quantisation overrides, resident
safetensors, per-layer ECB expert files) loads into decoder layers with the
reference's names, widths, head shapes, RoPE settings and K == V rule."""
import json
import os

import numpy as np
import pytest
import torch

import oracle

H, HD, GHD, I, E, IE, V = 128, 64, 128, 128, 4, 64, 256


def _bf(u16):
    return torch.from_numpy(np.ascontiguousarray(u16).view(np.int16)).view(torch.bfloat16)


def _qlin(t, prefix, out_f, in_f, bits, rng, names=(".scales", ".biases")):
    wq, s, b = oracle.quantize(rng.standard_normal((out_f, in_f)).astype(np.float32) * 0.05, bits)
    t[f"{prefix}.weight"] = wq
    t[prefix + names[0]] = _bf(s)
    t[prefix + names[1]] = _bf(b)


def _norm(n, rng):
    return torch.from_numpy(rng.standard_normal(n).astype(np.float32)).to(torch.bfloat16)


@pytest.fixture(scope="module")
def split_dir(fm, tmp_path_factory):
    d = tmp_path_factory.mktemp("split")
    rng = np.random.default_rng(0)
    args = {"hidden_size": H, "num_hidden_layers": 2, "num_attention_heads": 2, "num_key_value_heads": 2,
            "head_dim": HD, "vocab_size": V, "rms_norm_eps": 1e-6, "intermediate_size": I, "num_experts": E,
            "moe_intermediate_size": IE, "top_k_experts": 2, "layer_types": ["sliding_attention", "full_attention"],
            "global_head_dim": GHD, "num_global_key_value_heads": 1, "attention_k_eq_v": True,
            "final_logit_softcapping": 30.0, "sliding_window": 512,
            "rope_parameters": {"sliding_attention": {"rope_theta": 10000.0},
                                "full_attention": {"rope_theta": 1000000.0, "partial_rotary_factor": 0.25}}}
    quant = {"bits": 4, "group_size": 64, "mode": "affine",
             "language_model.model.embed_tokens": {"bits": 6, "group_size": 64}}
    for i in range(2):
        for p in ("q_proj", "v_proj"):
            quant[f"language_model.model.layers.{i}.self_attn.{p}"] = {"bits": 8, "group_size": 64}
    with open(d / "config.json", "w") as f:
        json.dump({"text_config": args, "quantization": quant}, f)
    t = {}
    for i, full in enumerate([False, True]):
        pre, hd = f"language_model.layers.{i}", GHD if full else HD
        kv = 1 if full else 2
        names = (".weight_scales", ".weight_biases") if full else (".scales", ".biases")  # both namings
        _qlin(t, f"{pre}.self_attn.q_proj", 2 * hd, H, 8, rng, names)
        _qlin(t, f"{pre}.self_attn.k_proj", kv * hd, H, 8, rng, names)
        if not full:
            _qlin(t, f"{pre}.self_attn.v_proj", kv * hd, H, 8, rng)
        _qlin(t, f"{pre}.self_attn.o_proj", H, 2 * hd, 8, rng, names)
        t[f"{pre}.self_attn.q_norm.weight"] = _norm(hd, rng)
        t[f"{pre}.self_attn.k_norm.weight"] = _norm(hd, rng)
        for n in ("input_layernorm", "post_attention_layernorm", "pre_feedforward_layernorm",
                  "post_feedforward_layernorm", "post_feedforward_layernorm_1", "post_feedforward_layernorm_2",
                  "pre_feedforward_layernorm_2"):
            t[f"{pre}.{n}.weight"] = _norm(H, rng)
        for p, (o, n) in {"gate_proj": (I, H), "up_proj": (I, H), "down_proj": (H, I)}.items():
            _qlin(t, f"{pre}.mlp.{p}", o, n, 4, rng)
        t[f"{pre}.router.proj.weight"] = _norm(E * H, rng).reshape(E, H)  # a bf16 router
        t[f"{pre}.router.scale"] = _norm(H, rng)
        t[f"{pre}.router.per_expert_scale"] = _norm(E, rng)
        t[f"{pre}.layer_scalar"] = torch.tensor([0.75], dtype=torch.bfloat16)
        offs, sizes, stride = fm.ecb_layout(H, IE)
        buf = torch.from_numpy(rng.integers(0, 255, E * stride, dtype=np.uint8))
        os.makedirs(d / "experts", exist_ok=True)
        fm.ecb.write(str(d / "experts" / f"layer_{i:02d}_experts.ecb"), fm.ExpertTable(buf, E, H, IE, 4, 64))
    _qlin(t, "language_model.embed_tokens", V, H, 6, rng)
    t["language_model.norm.weight"] = _norm(H, rng)
    os.makedirs(d / "resident")
    fm.safetensors.save(str(d / "resident" / "resident.safetensors"), t)
    return str(d), t


def test_split_layers(fm, split_dir):
    path, t = split_dir
    cfg, embed, layers, final_norm = fm.split.load_split(path, device="cpu")
    assert cfg["layer_full"] == [False, True] and cfg["window"] == 512 and cfg["softcap"] == 30.0
    assert (embed.bits, embed.in_features, embed.out_features) == (6, H, V)
    assert torch.equal(final_norm, t["language_model.norm.weight"])
    s, f = layers
    assert not s.k_eq_v and s.v_proj is not None and s.head_dim == HD and s.num_kv_heads == 2
    assert (s.rope_dims, s.rope_theta) == (HD, 10000.0) and not s.full_attention
    assert f.k_eq_v and f.v_proj is None and f.head_dim == GHD and f.num_kv_heads == 1 and f.full_attention
    assert (f.rope_dims, f.rope_theta) == (GHD // 4, 1e6)
    for L in layers:
        # k / o take the q_proj width of their layer (the reference keys attention on q_proj)
        assert L.q_proj.bits == 8 and L.k_proj.bits == 8 and L.o_proj.bits == 8
        assert L.mlp[0].bits == 4 and L.router["proj"].bits == 16
        assert L.layer_scalar == 0.75 and L.top_k == 2 and L.experts.num_experts == E
    assert s.v_proj.bits == 8  # v_proj has its own override
    assert torch.equal(s.norms["pre_ff_2"], t["language_model.layers.0.pre_feedforward_layernorm_2.weight"])
    assert torch.equal(f.q_proj.scales, t["language_model.layers.1.self_attn.q_proj.weight_scales"])


def test_model_cfg_global_kv_heads_follow_k_eq_v(fm, split_dir):
    """num_global_key_value_heads sizes the full layers' KV heads only when
    attention_k_eq_v is set (src/model/mod.rs:463); otherwise they keep
    num_key_value_heads, as load_split's layers do."""
    path, _ = split_dir
    args, _ = fm.split.read_config(path)
    assert fm.split.model_cfg(args, 6)["full_kv_heads"] == 1
    off = dict(args, attention_k_eq_v=False)
    assert fm.split.model_cfg(off, 6)["full_kv_heads"] == args["num_key_value_heads"] == 2


def test_split_expert_slice_and_missing_tensor(fm, split_dir, tmp_path):
    path, t = split_dir
    _, _, layers, _ = fm.split.load_split(path, device="cpu", n_layers=1, experts=(1, 2))
    assert (layers[0].experts.first_expert, layers[0].experts.num_experts) == (2, 2)
    q = fm.split.QuantConfig(None)
    assert q.bits_for("anything") == (8, 32)  # the reference's defaults without a quantization block
    q = fm.split.QuantConfig({"bits": 4, "group_size": 64, "x.q_proj": {"bits": 8, "group_size": 64}, "mode": "a"})
    assert q.bits_for("x.q_proj") == (8, 64) and q.bits_for("x.k_proj") == (4, 64)
    broken = dict(t)
    del broken["language_model.layers.0.router.scale"]
    bdir = tmp_path / "b"
    os.makedirs(bdir / "resident")
    os.symlink(os.path.join(path, "experts"), bdir / "experts")
    os.symlink(os.path.join(path, "config.json"), bdir / "config.json")
    fm.safetensors.save(str(bdir / "resident" / "resident.safetensors"), broken)
    with pytest.raises(KeyError, match="router.scale"):
        fm.split.load_split(str(bdir), device="cpu", n_layers=1)


_NAME_OF_CODE = {0: "U8", 1: "U32", 2: "BF16", 3: "F16", 4: "F32", 5: "I32"}


def _stacked_from_ecb(fm, path):
    """An ECB file's 9 tensors as expert-stacked (dtype, (E, *shape), bytes)."""
    hdr = fm.ecb.read_header(path)
    E, stride = hdr["num_experts"], hdr["stride"]
    with open(path, "rb") as f:
        f.seek(hdr["header_size"])
        data = np.frombuffer(f.read(E * stride), np.uint8).reshape(E, stride)
    out, off = [], 0
    for size, code, shape in hdr["tensors"]:
        out.append((_NAME_OF_CODE[code], (E,) + tuple(shape), data[:, off:off + size].tobytes()))
        off += size
    return out


def _checkpoint(fm, split_path, t, out, fused):
    """The fixture as an MLX checkpoint (two shards + index) in the UD or the fused layout."""
    st = fm.safetensors
    os.makedirs(out)
    res = {}
    for name, v in t.items():
        raw = st.read_raw(os.path.join(split_path, "resident", "resident.safetensors"), [name])[name]
        res[("model." + name) if fused else name.replace("language_model.", "language_model.model.", 1)] = raw
    exp = {}
    for i in range(2):
        s = _stacked_from_ecb(fm, os.path.join(split_path, "experts", f"layer_{i:02d}_experts.ecb"))
        if fused:
            pre = f"model.language_model.layers.{i}.experts"
            for j, suf in enumerate(("", "_scales", "_biases")):
                g, u = s[j], s[3 + j]
                E = g[1][0]
                gu = np.concatenate([np.frombuffer(g[2], np.uint8).reshape(E, -1),
                                     np.frombuffer(u[2], np.uint8).reshape(E, -1)], axis=1)
                exp[f"{pre}.gate_up_proj{suf}"] = (g[0], (E, 2 * g[1][1]) + g[1][2:], gu.tobytes())
                exp[f"{pre}.down_proj{suf}"] = s[6 + j]
        else:
            pre = f"language_model.model.layers.{i}.experts.switch_glu"
            for j, (p, c) in enumerate((p, c) for p in ("gate_proj", "up_proj", "down_proj")
                                       for c in ("weight", "scales", "biases")):
                exp[f"{pre}.{p}.{c}"] = s[j]
    st.save_raw(os.path.join(out, "model-00001-of-00002.safetensors"), res)
    st.save_raw(os.path.join(out, "model-00002-of-00002.safetensors"), exp)
    wm = {n: "model-00001-of-00002.safetensors" for n in res} | {n: "model-00002-of-00002.safetensors" for n in exp}
    with open(os.path.join(out, "model.safetensors.index.json"), "w") as f:
        json.dump({"metadata": {}, "weight_map": wm}, f)
    with open(os.path.join(split_path, "config.json")) as f, open(os.path.join(out, "config.json"), "w") as g:
        g.write(f.read())


@pytest.mark.parametrize("fused", [False, True])
def test_split_checkpoint_round_trip(fm, split_dir, tmp_path, fused):
    """An MLX checkpoint (Unsloth UD or mlx-community fused gate_up layout) split by
    split_checkpoint gives byte-identical ECB files and the same decoder layers as
    the split directory it was made from."""
    path, t = split_dir
    ckpt, out = str(tmp_path / "ckpt"), str(tmp_path / "out")
    _checkpoint(fm, path, t, ckpt, fused)
    meta = fm.split.split_checkpoint(ckpt, out)
    assert meta["layout"] == ("fused" if fused else "ud") and meta["num_expert_layers"] == 2
    for i in range(2):
        name = f"layer_{i:02d}_experts.ecb"
        with open(os.path.join(path, "experts", name), "rb") as a, open(os.path.join(out, "experts", name), "rb") as b:
            assert a.read() == b.read()
    _, e1, l1, n1 = fm.split.load_split(path, device="cpu")
    _, e2, l2, n2 = fm.split.load_split(out, device="cpu")
    assert torch.equal(e1.weight, e2.weight) and torch.equal(n1, n2)
    for a, b in zip(l1, l2):
        assert torch.equal(a.q_proj.weight, b.q_proj.weight) and torch.equal(a.mlp[2].scales, b.mlp[2].scales)
        assert torch.equal(a.router["per_expert_scale"], b.router["per_expert_scale"])
        assert torch.equal(a.experts.buf, b.experts.buf)
