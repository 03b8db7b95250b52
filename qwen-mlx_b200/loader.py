"""Weight loader for the reference's checkpoint layout (the GDN layers; the attention and MoE layers at the end).

The reference loads a Qwen3.5 MLX checkpoint in `load_config` / `load_model` (src/models/qwen3_5.rs:886-1086):

* `config.json`, whose fields may sit under `text_config` (merged over the top level, qwen3_5.rs:888-909), with
  an optional `quantization: {group_size, bits}` block (qwen3_5.rs:915-925);
* safetensors shards listed by `model.safetensors.index.json` (`weight_map`), or one `model.safetensors`
  (qwen3_5.rs:940-955);
* per linear-attention layer l (`(l + 1) % full_attention_interval != 0`, qwen3_5.rs:73-75), tensors named
  `language_model.model.layers.{l}.linear_attn.{in_proj_qkv, in_proj_z, in_proj_a, in_proj_b, out_proj}`
  (`.weight`, plus `.scales` / `.biases` when quantized: MLX affine, `.weight` holding uint32 words of 4-bit
  codes), `.conv1d.weight` [D, K, 1], `.norm.weight` [dv], `.A_log`, `.dt_bias` [Hv], and the decoder layer's
  `input_layernorm.weight` [hidden] (qwen3_5.rs:463-503, :675-720);
* at load the reference merges `[qkv; z]` and `[b; a]` by rows (qwen3_5.rs:1024-1057) and re-lays the conv weight
  (qwen3_5.rs:1058-1066); norm weights are used as stored (pre-shifted in these checkpoints, qwen3_5.rs:975).

This module reads the same files (a self-contained safetensors reader: 8-byte little-endian header length,
JSON header of `{name: {dtype, shape, data_offsets}}`, raw little-endian data) and returns, per GDN layer, the
weight dict the rest of the package uses: `conv_w` [D, K] bf16, `A_log`, `dt_bias` f32, `norm_w`, `pre_w` bf16,
and either bf16 `w_qkv`, `w_z`, `w_b`, `w_a`, `w_out` or, for a quantized checkpoint, `q4_in` / `q4_out` =
(w_q uint32, scales, biases) with the in-projection rows merged in the order `[qkv; z; b; a]` (the reference's
`[qkv; z]` then `[b; a]`).  bf16 tensors are numpy uint16 bit patterns.  A_log and dt_bias are widened to f32
(exactly), and `dt_bias_bf16` records whether the checkpoint stores dt_bias in bf16: the reference then adds
`a + dt_bias` and takes its exp as bf16 ops (compiled_ops.rs:36-37), and the kernels and the oracle reproduce those
two roundings when the flag is set.  (A_log is cast to f32 by the reference itself, :41, so its dtype changes
nothing.)
"""
from __future__ import annotations

import json
import struct
from pathlib import Path

import numpy as np

from .synth import GdnConfig, f32_to_bf16

_DTYPES = {"BF16": np.uint16, "F16": np.float16, "F32": np.float32, "U32": np.uint32, "I32": np.int32,
           "U8": np.uint8, "I8": np.int8, "U16": np.uint16, "I64": np.int64, "F64": np.float64}
PREFIX = "language_model.model.layers"


class SafeTensors:
    """Read-only view of one .safetensors file (memory-mapped)."""

    def __init__(self, path):
        self.path = Path(path)
        with open(self.path, "rb") as f:
            (n,) = struct.unpack("<Q", f.read(8))
            header = json.loads(f.read(n))
        self.meta = {k: v for k, v in header.items() if k != "__metadata__"}
        self._base = 8 + n
        self._mm = np.memmap(self.path, dtype=np.uint8, mode="r")

    def keys(self):
        return self.meta.keys()

    def dtype(self, name: str) -> str:
        return self.meta[name]["dtype"]

    def get(self, name: str) -> np.ndarray:
        m = self.meta[name]
        if m["dtype"] not in _DTYPES:
            raise ValueError(f"{self.path.name}: tensor {name} has unsupported dtype {m['dtype']}")
        b0, b1 = m["data_offsets"]
        raw = self._mm[self._base + b0:self._base + b1]
        return np.frombuffer(bytearray(raw), dtype=_DTYPES[m["dtype"]]).reshape(m["shape"])  # writable copy


def save_safetensors(path, tensors: dict, bf16: set = frozenset()):
    """Write a .safetensors file (used to make test checkpoints).  Names in `bf16` are uint16 bit patterns
    stored with dtype BF16."""
    inv = {np.dtype(np.float16): "F16", np.dtype(np.float32): "F32", np.dtype(np.uint32): "U32",
           np.dtype(np.int32): "I32", np.dtype(np.uint8): "U8", np.dtype(np.uint16): "U16"}
    header, blobs, off = {}, [], 0
    for name, arr in tensors.items():
        arr = np.ascontiguousarray(arr)
        dt = "BF16" if name in bf16 else inv[arr.dtype]
        b = arr.tobytes()
        header[name] = {"dtype": dt, "shape": list(arr.shape), "data_offsets": [off, off + len(b)]}
        blobs.append(b)
        off += len(b)
    h = json.dumps(header).encode()
    h += b" " * ((8 - len(h) % 8) % 8)
    with open(path, "wb") as f:
        f.write(struct.pack("<Q", len(h)))
        f.write(h)
        for b in blobs:
            f.write(b)


def load_config(model_dir) -> dict:
    """config.json with `text_config` merged over the top level (top-level keys fill in missing ones)."""
    raw = json.loads((Path(model_dir) / "config.json").read_text())
    if "text_config" in raw:
        cfg = dict(raw["text_config"])
        for k, v in raw.items():
            if k not in ("text_config", "vision_config"):
                cfg.setdefault(k, v)
        return cfg
    return raw


def gdn_config(cfg: dict) -> GdnConfig:
    """The GDN shapes of a checkpoint config (n_layers = the number of linear-attention layers)."""
    return GdnConfig(hidden=cfg["hidden_size"], n_k_heads=cfg["linear_num_key_heads"],
                     n_v_heads=cfg["linear_num_value_heads"], head_k_dim=cfg["linear_key_head_dim"],
                     head_v_dim=cfg["linear_value_head_dim"], conv_kernel=cfg.get("linear_conv_kernel_dim", 4),
                     n_layers=len(linear_layers(cfg)), rms_norm_eps=cfg["rms_norm_eps"])


def linear_layers(cfg: dict) -> list[int]:
    """Indices of the linear-attention (GDN) layers: (l + 1) % full_attention_interval != 0."""
    n, k = cfg["num_hidden_layers"], cfg["full_attention_interval"]
    return [l for l in range(n) if (l + 1) % k != 0]


class Checkpoint:
    """All tensors of a checkpoint directory, by name, across its shards."""

    def __init__(self, model_dir):
        d = Path(model_dir)
        index = d / "model.safetensors.index.json"
        if index.exists():
            files = sorted(set(json.loads(index.read_text())["weight_map"].values()))
        else:
            files = ["model.safetensors"]
        self.files = [SafeTensors(d / f) for f in files]
        self.where = {}
        for st in self.files:
            for k in st.keys():
                self.where[k] = st

    def __contains__(self, name):
        return name in self.where

    def get(self, name: str) -> np.ndarray:
        if name not in self.where:
            raise KeyError(f"checkpoint has no tensor {name}")
        return self.where[name].get(name)

    def dtype(self, name: str) -> str:
        return self.where[name].dtype(name)


def _bf16(ck: Checkpoint, name: str) -> np.ndarray:
    a = ck.get(name)
    dt = ck.dtype(name)
    if dt == "BF16":
        return a
    if dt in ("F16", "F32", "F64"):
        return f32_to_bf16(a.astype(np.float32))
    raise ValueError(f"{name}: expected a floating tensor, got {dt}")


def _f32(ck: Checkpoint, name: str) -> np.ndarray:
    a = ck.get(name)
    if ck.dtype(name) == "BF16":
        return (a.astype(np.uint32) << np.uint32(16)).view(np.float32)
    return a.astype(np.float32)


def _proj(ck: Checkpoint, base: str, quantized: bool, bits: int, group: int):
    """One projection: bf16 weight [N, K], or (w_q uint32 [N, K/8], scales, biases [N, K/group]) for a
    quantized one (MLX affine)."""
    if quantized and base + ".scales" in ck:
        if bits != 4 or group != 64:
            raise ValueError(f"{base}: {bits}-bit group-{group} quantization; the kernels take bits 4, group 64")
        return (np.ascontiguousarray(ck.get(base + ".weight"), np.uint32), _bf16(ck, base + ".scales"),
                _bf16(ck, base + ".biases"))
    return _bf16(ck, base + ".weight")


def load_gdn_layers(model_dir) -> tuple[GdnConfig, list[int], list[dict]]:
    """(GDN shapes, linear-layer indices, one weight dict per GDN layer) of a checkpoint directory."""
    cfg = load_config(model_dir)
    q = cfg.get("quantization")
    quantized = q is not None
    bits = int(q.get("bits", 4)) if q else 4
    group = int(q.get("group_size", 64)) if q else 64
    g = gdn_config(cfg)
    ck = Checkpoint(model_dir)
    layers = linear_layers(cfg)
    out = []
    for l in layers:
        p = f"{PREFIX}.{l}.linear_attn"
        conv = _bf16(ck, f"{p}.conv1d.weight")
        if conv.ndim == 3:
            conv = conv.reshape(conv.shape[0], conv.shape[1])   # [D, K, 1] -> [D, K]
        w = {
            "conv_w": np.ascontiguousarray(conv),
            "A_log": _f32(ck, f"{p}.A_log"),
            "dt_bias": _f32(ck, f"{p}.dt_bias"),
            "dt_bias_bf16": ck.dtype(f"{p}.dt_bias") == "BF16",
            "norm_w": _bf16(ck, f"{p}.norm.weight"),
            "pre_w": _bf16(ck, f"{PREFIX}.{l}.input_layernorm.weight"),
        }
        parts = {name: _proj(ck, f"{p}.{name}", quantized, bits, group)
                 for name in ("in_proj_qkv", "in_proj_z", "in_proj_b", "in_proj_a", "out_proj")}
        kinds = {isinstance(v, tuple) for v in parts.values()}
        if len(kinds) != 1:
            raise ValueError(f"layer {l}: some projections are quantized and some are not")
        if isinstance(parts["in_proj_qkv"], tuple):
            order = ("in_proj_qkv", "in_proj_z", "in_proj_b", "in_proj_a")     # [qkv; z] then [b; a]
            w["q4_in"] = tuple(np.concatenate([parts[n][i] for n in order], axis=0) for i in range(3))
            w["q4_out"] = parts["out_proj"]
        else:
            w["w_qkv"], w["w_z"] = parts["in_proj_qkv"], parts["in_proj_z"]
            w["w_b"], w["w_a"], w["w_out"] = parts["in_proj_b"], parts["in_proj_a"], parts["out_proj"]
        _check_shapes(g, w, l)
        out.append(w)
    return g, layers, out


def _check_shapes(g: GdnConfig, w: dict, l: int):
    D, H, Z = g.conv_dim, g.hidden, g.z_dim
    want = {"conv_w": (D, g.conv_k), "A_log": (g.hv,), "dt_bias": (g.hv,), "norm_w": (g.dv,), "pre_w": (H,)}
    if "q4_in" in w:
        want.update({"q4_in": (D + Z + 2 * g.hv, H // 8), "q4_out": (H, Z // 8)})
    else:
        want.update({"w_qkv": (D, H), "w_z": (Z, H), "w_b": (g.hv, H), "w_a": (g.hv, H), "w_out": (H, Z)})
    for k, shape in want.items():
        got = w[k][0].shape if isinstance(w[k], tuple) else w[k].shape
        if tuple(got) != shape:
            raise ValueError(f"layer {l}: {k} has shape {tuple(got)}, expected {shape}")


# ---------------------------------------------------------------- attention and MoE layers
#
# The other layers of the hybrid decoder (qwen3_5.rs:313-460, :78-311) as the reference's checkpoint stores them:
#   language_model.model.layers.{l}.self_attn.{q_proj, k_proj, v_proj, o_proj}   (l + 1) % interval == 0
#       q_proj has 2 * n_heads * head_dim rows (queries and the output gate, per head), :345-350
#   language_model.model.layers.{l}.self_attn.{q_norm, k_norm}.weight [head_dim]
#   language_model.model.layers.{l}.post_attention_layernorm.weight [hidden]           every layer, :740
#   language_model.model.layers.{l}.mlp.gate                [E, hidden]                 the router, :241
#   language_model.model.layers.{l}.mlp.switch_mlp.{gate_proj, up_proj, down_proj}   [E, I, hidden], [E, hidden, I]
#   language_model.model.layers.{l}.mlp.shared_expert.{gate_proj, up_proj, down_proj}
#   language_model.model.layers.{l}.mlp.shared_expert_gate [1, hidden]
# A quantized checkpoint quantizes every one of them with the one (bits, group_size) of its config
# (nn::quantize over the whole model, qwen3_5.rs:927-935).

def attention_layers(cfg: dict) -> list[int]:
    """Indices of the full-attention layers: (l + 1) % full_attention_interval == 0 (qwen3_5.rs:73-75)."""
    n, k = cfg["num_hidden_layers"], cfg["full_attention_interval"]
    return [l for l in range(n) if (l + 1) % k == 0]


def attn_config(cfg: dict, max_ctx: int = 4096) -> dict:
    """Keyword arguments of hybrid.AttnConfig from a checkpoint config (defaults as Qwen35Config's, :67-68)."""
    hd = int(cfg["head_dim"])
    return dict(n_heads=int(cfg["num_attention_heads"]), n_kv_heads=int(cfg["num_key_value_heads"]), head_dim=hd,
                rotary_dim=int(hd * float(cfg.get("partial_rotary_factor", 0.25))),
                rope_theta=float(cfg.get("rope_theta", 10_000_000.0)), rms_norm_eps=float(cfg["rms_norm_eps"]),
                max_ctx=max_ctx)


def moe_config(cfg: dict) -> dict:
    """Keyword arguments of hybrid.MoeConfig from a checkpoint config (qwen3_5.rs:55-63)."""
    return dict(hidden=int(cfg["hidden_size"]), n_experts=int(cfg["num_experts"]),
                top_k=int(cfg["num_experts_per_tok"]), moe_inter=int(cfg["moe_intermediate_size"]),
                shared_inter=int(cfg["shared_expert_intermediate_size"]),
                norm_topk_prob=bool(cfg.get("norm_topk_prob", True)))


def dequantize(w_q: np.ndarray, scales: np.ndarray, biases: np.ndarray, bits: int, group: int) -> np.ndarray:
    """MLX affine dequantization to bf16: value c of a row = scale[c / group] * q + bias[c / group], q = bits
    [bits * (c % (32 / bits)), +bits) of word c / (32 / bits), rounded once (exact in f32 for bits <= 8, since a
    bf16 scale times a code and its bias are exact there)."""
    per = 32 // bits
    w_q = np.asarray(w_q, np.uint32)
    lead, W = w_q.shape[:-1], w_q.shape[-1]
    shifts = (np.arange(per, dtype=np.uint32) * bits)
    q = ((w_q[..., None] >> shifts) & np.uint32((1 << bits) - 1)).reshape(*lead, W * per).astype(np.float32)
    s = (np.asarray(scales, np.uint16).astype(np.uint32) << 16).view(np.float32)
    b = (np.asarray(biases, np.uint16).astype(np.uint32) << 16).view(np.float32)
    cols = W * per
    v = q.reshape(*lead, cols // group, group) * s[..., None] + b[..., None]
    return f32_to_bf16(v.reshape(*lead, cols).astype(np.float32))


def _quant(cfg: dict):
    q = cfg.get("quantization")
    if q is None:
        return None
    return int(q.get("bits", 4)), int(q.get("group_size", 64))


def _dense_bf16(ck: Checkpoint, base: str, quant) -> np.ndarray:
    """A Linear's weight as bf16, dequantizing a quantized one (the router and the shared-expert gate, which the
    kernels take in bf16)."""
    if quant is not None and base + ".scales" in ck:
        bits, group = quant
        return dequantize(ck.get(base + ".weight"), _bf16(ck, base + ".scales"), _bf16(ck, base + ".biases"), bits,
                          group)
    return _bf16(ck, base + ".weight")


def _q4_matrix(ck: Checkpoint, base: str, quant, rows: int, cols: int) -> dict:
    """A 4-bit (group 64) matrix as {q, scales, biases}, experts stacked by rows: [rows][cols/8] words."""
    if quant is None or base + ".scales" not in ck:
        raise ValueError(f"{base}: the MoE kernels take MLX 4-bit (group 64) experts; this tensor is not quantized")
    if quant != (4, 64):
        raise ValueError(f"{base}: {quant[0]}-bit group-{quant[1]} quantization; the kernels take bits 4, group 64")
    wq = ck.get(base + ".weight")
    if wq.shape[-1] != cols // 8 or wq.size != rows * (cols // 8):
        raise ValueError(f"{base}: weight of shape {wq.shape}, expected {rows} rows of {cols // 8} words")
    m = {"q": np.ascontiguousarray(wq, np.uint32).reshape(rows, cols // 8),
         "scales": _bf16(ck, base + ".scales").reshape(rows, cols // 64),
         "biases": _bf16(ck, base + ".biases").reshape(rows, cols // 64)}
    return m


def load_attention_layers(model_dir, max_ctx: int = 4096) -> tuple[dict, list[int], list[dict]]:
    """(hybrid.AttnConfig keyword arguments, attention-layer indices, one weight dict per attention layer):
    `q_proj` / `k_proj` / `v_proj` / `o_proj` (bf16 [N, K], or (w_q, scales, biases) when quantized; they run as
    library GEMMs around gdn_attn_step), `q_norm_w` / `k_norm_w` [head_dim], `pre_w` (input_layernorm) and
    `post_w` (post_attention_layernorm) [hidden], all bf16."""
    cfg = load_config(model_dir)
    quant = _quant(cfg)
    bits, group = quant if quant else (4, 64)
    a = attn_config(cfg, max_ctx)
    H, nh, nkv, hd = int(cfg["hidden_size"]), a["n_heads"], a["n_kv_heads"], a["head_dim"]
    ck = Checkpoint(model_dir)
    layers = attention_layers(cfg)
    want = {"q_proj": (2 * nh * hd, H), "k_proj": (nkv * hd, H), "v_proj": (nkv * hd, H), "o_proj": (H, nh * hd)}
    out = []
    for l in layers:
        p = f"{PREFIX}.{l}.self_attn"
        w = {name: _proj(ck, f"{p}.{name}", quant is not None, bits, group) for name in want}
        for name, (n, k) in want.items():
            got = w[name][0].shape if isinstance(w[name], tuple) else w[name].shape
            exp = (n, k // 8) if isinstance(w[name], tuple) else (n, k)
            if tuple(got) != exp:
                raise ValueError(f"layer {l}: {name} has shape {tuple(got)}, expected {exp}")
        w["q_norm_w"] = _bf16(ck, f"{p}.q_norm.weight")
        w["k_norm_w"] = _bf16(ck, f"{p}.k_norm.weight")
        w["pre_w"] = _bf16(ck, f"{PREFIX}.{l}.input_layernorm.weight")
        w["post_w"] = _bf16(ck, f"{PREFIX}.{l}.post_attention_layernorm.weight")
        for k, n in (("q_norm_w", hd), ("k_norm_w", hd), ("pre_w", H), ("post_w", H)):
            if w[k].shape != (n,):
                raise ValueError(f"layer {l}: {k} has shape {w[k].shape}, expected ({n},)")
        out.append(w)
    return a, layers, out


def load_moe_layers(model_dir) -> tuple[dict, list[dict]]:
    """(hybrid.MoeConfig keyword arguments, one hybrid.MoeWeights input dict per decoder layer): `router` [E,
    hidden] and `shared_gate` [hidden] bf16 (dequantized when the checkpoint quantizes them), the experts'
    `gate` / `up` [E * I][hidden / 8] and `down` [E * hidden][I / 8] and the shared expert's `sh_gate` /
    `sh_up` / `sh_down` as 4-bit {q, scales, biases}, and `post_w` (post_attention_layernorm) [hidden]."""
    cfg = load_config(model_dir)
    quant = _quant(cfg)
    m = moe_config(cfg)
    H, E, I, Is = m["hidden"], m["n_experts"], m["moe_inter"], m["shared_inter"]
    ck = Checkpoint(model_dir)
    out = []
    for l in range(int(cfg["num_hidden_layers"])):
        p = f"{PREFIX}.{l}.mlp"
        w = {"router": _dense_bf16(ck, f"{p}.gate", quant),
             "shared_gate": _dense_bf16(ck, f"{p}.shared_expert_gate", quant).reshape(-1),
             "gate": _q4_matrix(ck, f"{p}.switch_mlp.gate_proj", quant, E * I, H),
             "up": _q4_matrix(ck, f"{p}.switch_mlp.up_proj", quant, E * I, H),
             "down": _q4_matrix(ck, f"{p}.switch_mlp.down_proj", quant, E * H, I),
             "sh_gate": _q4_matrix(ck, f"{p}.shared_expert.gate_proj", quant, Is, H),
             "sh_up": _q4_matrix(ck, f"{p}.shared_expert.up_proj", quant, Is, H),
             "sh_down": _q4_matrix(ck, f"{p}.shared_expert.down_proj", quant, H, Is),
             "post_w": _bf16(ck, f"{PREFIX}.{l}.post_attention_layernorm.weight")}
        if w["router"].shape != (E, H) or w["shared_gate"].shape != (H,):
            raise ValueError(f"layer {l}: router {w['router'].shape} / shared_expert_gate {w['shared_gate'].shape}, "
                             f"expected ({E}, {H}) / ({H},)")
        out.append(w)
    return m, out
