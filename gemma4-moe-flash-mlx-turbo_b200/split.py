"""Loading a split Gemma-4 checkpoint: the reference's load_gemma4_model
(src/model/mod.rs:405-617) for this library's decoder.

    <split>/config.json                     TextModelArgs ("text_config" or the top level)
                                            and "quantization" (src/config.rs:13-37, 97-235)
    <split>/resident/resident.safetensors   every tensor but the routed experts
    <split>/experts/layer_XX_experts.ecb    each layer's routed experts (src/memory.rs:386-398)

split_checkpoint() makes that layout from an MLX checkpoint (the reference's
splitter, src/splitter.rs:99-196); load_split() returns (cfg, embed, layers,
final_norm) for Gemma4Model(cfg, embed,
layers, final_norm, batch, max_positions, ...).  Names, per-component bit widths
(overrides keyed by "language_model.model.layers.N.<component>") and the
flexible scale / bias names follow the reference; quantised linears whose width
or group the kernels do not serve are re-quantised at load (safetensors.load_qlinear,
on the GPU).  The routed experts must be 4-bit, group 64 (the expert kernels).
"""
from __future__ import annotations

import json
import os
import re
import shutil

import numpy as np

from . import ecb as _ecb
from . import safetensors as _st
from .model import Gemma4DecoderLayer


class QuantConfig:
    """config.json "quantization": global bits / group_size and per-weight
    overrides {path: {"bits", "group_size"}} (src/config.rs:13-75)."""

    def __init__(self, q: dict | None):
        q = q or {}
        self.present = bool(q)
        self.bits = int(q.get("bits", 4))
        self.group_size = int(q.get("group_size", 64))
        self.overrides = {k: v for k, v in q.items()
                          if k not in ("bits", "group_size", "mode") and isinstance(v, dict) and "bits" in v}

    def bits_for(self, path: str) -> tuple[int, int]:
        if not self.present:  # no quantization block: the reference's defaults (mod.rs:417-418)
            return 8, 32
        o = self.overrides.get(path, {})
        return int(o.get("bits", self.bits)), int(o.get("group_size", self.group_size))


def read_config(split_dir: str) -> tuple[dict, QuantConfig]:
    with open(os.path.join(split_dir, "config.json")) as f:
        config = json.load(f)
    return config.get("text_config", config), QuantConfig(config.get("quantization"))


def rope_config(args: dict, full: bool) -> tuple[int, float]:
    """(rotated dims, theta) of a layer type (TextModelArgs::gemma4_rope_config, config.rs:212-227)."""
    p = (args.get("rope_parameters") or {}).get("full_attention" if full else "sliding_attention") or {}
    theta = float(p.get("rope_theta", 10000.0))
    partial = float(p.get("partial_rotary_factor", 1.0))
    head_dim = (args.get("global_head_dim") or args["head_dim"]) if full else args["head_dim"]
    return int(head_dim * partial), theta


def model_cfg(args: dict, embed_bits: int) -> dict:
    """The decoder's config dict (the keys Gemma4Model and bench use) from TextModelArgs."""
    types = args["layer_types"]
    full = [t == "full_attention" for t in types]
    fr = rope_config(args, True)
    sr = rope_config(args, False)
    return dict(hidden=args["hidden_size"], layers=args["num_hidden_layers"], heads=args["num_attention_heads"],
                sliding_kv_heads=args["num_key_value_heads"], sliding_head_dim=args["head_dim"],
                full_kv_heads=(args.get("num_global_key_value_heads") or args["num_key_value_heads"])
                if args.get("attention_k_eq_v") else args["num_key_value_heads"],
                full_head_dim=args.get("global_head_dim") or args["head_dim"], sliding_theta=sr[1],
                full_theta=fr[1], full_partial_rotary=fr[0] / (args.get("global_head_dim") or args["head_dim"]),
                window=args.get("sliding_window") or 1024, dense_inter=args.get("intermediate_size"),
                experts=args["num_experts"], expert_inter=args["moe_intermediate_size"],
                top_k=args.get("top_k_experts") or args.get("num_experts_per_tok") or 8, vocab=args["vocab_size"],
                eps=args["rms_norm_eps"], softcap=args.get("final_logit_softcapping") or 0.0, embed_bits=embed_bits,
                layer_full=full)


def _qlin(weights, prefix, bits_gs):
    return _st.load_qlinear(weights, prefix, bits_gs[0], bits_gs[1])


def load_split(split_dir: str, device="cuda", n_layers: int | None = None, experts: tuple[int, int] | None = None):
    """-> (cfg, embed QuantizedLinear, [Gemma4DecoderLayer], final_norm bf16).
    experts = (rank, world) keeps one rank's contiguous expert slice per layer."""
    args, quant = read_config(split_dir)
    weights = _st.load(os.path.join(split_dir, "resident", "resident.safetensors"), device=device)

    def get(name):
        if name not in weights:
            raise KeyError(f"missing weight: {name}")
        return weights[name]

    n = args["num_hidden_layers"] if n_layers is None else n_layers
    H, eps = args["hidden_size"], args["rms_norm_eps"]
    top_k = args.get("top_k_experts") or args.get("num_experts_per_tok") or 8
    layers = []
    for i in range(n):
        pre, cfgp = f"language_model.layers.{i}", f"language_model.model.layers.{i}"
        full = args["layer_types"][i] == "full_attention"
        k_eq_v = bool(args.get("attention_k_eq_v")) and full
        head_dim = (args.get("global_head_dim") or args["head_dim"]) if full else args["head_dim"]
        kv_heads = (args.get("num_global_key_value_heads") or args["num_key_value_heads"]) if k_eq_v \
            else args["num_key_value_heads"]
        rope_dims, theta = rope_config(args, full)
        a = f"{pre}.self_attn"
        ab = quant.bits_for(f"{cfgp}.self_attn.q_proj")
        q, k, o = (_qlin(weights, f"{a}.{p}", ab) for p in ("q_proj", "k_proj", "o_proj"))
        v = None if k_eq_v else _qlin(weights, f"{a}.v_proj", quant.bits_for(f"{cfgp}.self_attn.v_proj"))
        norms = {"input": get(f"{pre}.input_layernorm.weight"),
                 "post_attn": get(f"{pre}.post_attention_layernorm.weight"),
                 "pre_ff": get(f"{pre}.pre_feedforward_layernorm.weight"),
                 "post_ff_1": get(f"{pre}.post_feedforward_layernorm_1.weight"),
                 "pre_ff_2": get(f"{pre}.pre_feedforward_layernorm_2.weight"),
                 "post_ff_2": get(f"{pre}.post_feedforward_layernorm_2.weight"),
                 "post_ff": get(f"{pre}.post_feedforward_layernorm.weight")}
        mb = quant.bits_for(f"{cfgp}.mlp.gate_proj")
        mlp = tuple(_qlin(weights, f"{pre}.mlp.{p}", mb) for p in ("gate_proj", "up_proj", "down_proj"))
        router = {"proj": _qlin(weights, f"{pre}.router.proj", quant.bits_for(f"{cfgp}.router.proj")),
                  "router_scale": get(f"{pre}.router.scale"),
                  "per_expert_scale": get(f"{pre}.router.per_expert_scale"), "root_size": H ** -0.5}
        path = os.path.join(split_dir, "experts", f"layer_{i:02d}_experts.ecb")
        if experts is None:
            table = _ecb.load(path, device=device)
        else:
            hdr = _ecb.read_header(path)
            E, (r, w) = hdr["num_experts"], experts
            table = _ecb.load(path, device=device, experts=(r * (E // w), E // w))
        if (table.bits, table.group) != (4, 64):
            raise ValueError(f"{path}: {table.bits}-bit, group {table.group} experts (the expert kernels: 4-bit, "
                             f"group 64)")
        ls = weights.get(f"{pre}.layer_scalar")
        layer = Gemma4DecoderLayer(q, k, v, o, get(f"{a}.q_norm.weight"), get(f"{a}.k_norm.weight"), norms, mlp,
                                   router, table, args["num_attention_heads"], kv_heads, head_dim, rope_dims, theta,
                                   k_eq_v, eps=eps, layer_scalar=1.0 if ls is None else float(ls.float().item()),
                                   attn_scale=1.0, top_k=top_k)
        layer.full_attention = full
        layers.append(layer)
    eb, egs = quant.bits_for("language_model.model.embed_tokens")
    ew = get("language_model.embed_tokens.weight")
    es = weights.get("language_model.embed_tokens.scales", weights.get("language_model.embed_tokens.weight_scales"))
    if es is None:
        raise ValueError("bf16 embedding: the lm_head kernels serve 4 / 6 / 8-bit tables; quantise it first")
    embed = _st.load_qlinear({"e.weight": ew, "e.scales": es,
                              "e.biases": weights.get("language_model.embed_tokens.biases",
                                                      weights.get("language_model.embed_tokens.weight_biases"))},
                             "e", eb, egs)
    cfg = model_cfg(args, embed.bits)
    return cfg, embed, layers, get("language_model.norm.weight")


_CONFIG_FILES = ("config.json", "tokenizer.json", "tokenizer_config.json", "generation_config.json",
                 "chat_template.jinja")
_PROJ, _COMP = ("gate_proj", "up_proj", "down_proj"), ("weight", "scales", "biases")


def _layout(names) -> str:
    """'ud' (Unsloth: language_model.model.layers.N.experts.switch_glu.<proj>.<comp>) or
    'fused' (mlx-community: model.language_model.layers.N.experts.{gate_up_proj,down_proj}[_scales|_biases]),
    src/splitter.rs:24-38 for the Gemma-4 layouts."""
    if any(".experts.switch_glu." in n for n in names):
        return "ud"
    if any(".experts.gate_up_proj" in n or ".experts.down_proj" in n for n in names):
        return "fused"
    raise ValueError("no Gemma-4 expert tensors (experts.switch_glu.* or experts.gate_up_proj / down_proj)")


def _is_expert(name: str, layout: str) -> bool:
    return ".experts.switch_glu." in name if layout == "ud" else (".experts.gate_up_proj" in name
                                                                   or ".experts.down_proj" in name)


def _canonical(name: str, layout: str) -> str:
    """Resident names start with language_model.layers.N / language_model.embed_tokens
    (src/splitter.rs:80-95)."""
    if layout == "ud":
        return name.replace("language_model.model.", "language_model.", 1)
    return name[len("model."):] if name.startswith("model.") else name


def _stacked(raw) -> tuple[str, tuple, np.ndarray]:
    """(dtype, per-expert shape, uint8 [E, per-expert bytes]) of an expert-stacked tensor."""
    dt, shape, data = raw
    E = shape[0]
    return dt, tuple(shape[1:]), np.frombuffer(data, np.uint8).reshape(E, -1)


def _halves(t):
    """Split a fused gate_up tensor along its first per-expert dim: (gate, up)
    (src/splitter.rs:362-403)."""
    dt, shape, a = t
    if shape[0] % 2:
        raise ValueError(f"fused gate_up dim {shape[0]} is odd")
    h = a.shape[1] // 2
    half = (shape[0] // 2,) + tuple(shape[1:])
    return (dt, half, a[:, :h]), (dt, half, a[:, h:])


def split_checkpoint(model_dir: str, out_dir: str) -> dict:
    """MLX checkpoint (model.safetensors.index.json + shards) -> split layout:
    resident/resident.safetensors (every non-expert tensor, canonical names),
    experts/layer_XX_experts.ecb (9 tensors per layer: gate / up / down x
    weight / scales / biases, expert-major), the config files and
    split_config.json.  Returns the split metadata."""
    with open(os.path.join(model_dir, "model.safetensors.index.json")) as f:
        weight_map = json.load(f)["weight_map"]
    layout = _layout(weight_map)
    os.makedirs(os.path.join(out_dir, "resident"), exist_ok=True)
    os.makedirs(os.path.join(out_dir, "experts"), exist_ok=True)
    for name in _CONFIG_FILES:
        if os.path.exists(os.path.join(model_dir, name)):
            shutil.copyfile(os.path.join(model_dir, name), os.path.join(out_dir, name))
    by_shard: dict[str, list[str]] = {}
    for name, shard in weight_map.items():
        by_shard.setdefault(shard, []).append(name)
    raw = {}
    for shard, names in sorted(by_shard.items()):
        raw.update(_st.read_raw(os.path.join(model_dir, shard), names))
    resident = {_canonical(n, layout): raw[n] for n in sorted(weight_map) if not _is_expert(n, layout)}
    _st.save_raw(os.path.join(out_dir, "resident", "resident.safetensors"), resident)
    pat = re.compile(r"layers\.(\d+)\.experts\.")
    n_layers = 1 + max(int(pat.search(n).group(1)) for n in weight_map if _is_expert(n, layout))
    for i in range(n_layers):
        if layout == "ud":
            pre = f"language_model.model.layers.{i}.experts.switch_glu"
            tensors = [_stacked(raw[f"{pre}.{p}.{c}"]) for p in _PROJ for c in _COMP]
        else:
            pre = f"model.language_model.layers.{i}.experts"
            gate, up = zip(*(_halves(_stacked(raw[f"{pre}.gate_up_proj{s}"])) for s in ("", "_scales", "_biases")))
            down = [_stacked(raw[f"{pre}.down_proj{s}"]) for s in ("", "_scales", "_biases")]
            tensors = list(gate) + list(up) + down
        _ecb.write_tensors(os.path.join(out_dir, "experts", f"layer_{i:02d}_experts.ecb"), tensors)
    meta = {"original_model": model_dir, "resident_dir": "resident", "expert_dir": "experts", "format": "ecb",
            "layout": layout, "num_expert_layers": n_layers}
    with open(os.path.join(out_dir, "split_config.json"), "w") as f:
        json.dump(meta, f, indent=2)
    return meta
