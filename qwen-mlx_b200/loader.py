"""Weight loader for the reference's checkpoint layout (the GDN layers only).

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
