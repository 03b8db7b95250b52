"""Seeded synthetic inputs and weights for the GDN layer step.

There is no checkpoint or dataset on the hot path: every parity test, golden
fixture and benchmark draws its tensors from this counter-based generator so
that the CUDA path, the CPU oracle and the CPU baseline see bit-identical
bytes.  The generator is SplitMix64 over (seed, stream-name, element index);
normals come from the Box-Muller cosine branch, one normal per two uniforms.
It is pure numpy and does not depend on numpy's own bit-generator streams, so
the bytes are stable across numpy versions.

Distributions follow the reference model's synthetic stand-in:
  * projection and conv weights  N(0, 0.02) bf16
  * A_log ~ U(log 1, log 16) f32, dt_bias ~ U(-1, 1) f32
  * RMSNorm gains = 1.0 (bf16)
  * token activations ~ N(0, 1) bf16
"""
from __future__ import annotations

import math
import numpy as np

_U64 = np.uint64
_GOLDEN = _U64(0x9E3779B97F4A7C15)
_M1 = _U64(0xBF58476D1CE4E5B9)
_M2 = _U64(0x94D049BB133111EB)


def splitmix64(x: np.ndarray) -> np.ndarray:
    """SplitMix64 finaliser applied elementwise to a uint64 array."""
    with np.errstate(over="ignore"):
        z = x + _GOLDEN
        z = (z ^ (z >> _U64(30))) * _M1
        z = (z ^ (z >> _U64(27))) * _M2
        return z ^ (z >> _U64(31))


def _fnv1a64(name: str) -> int:
    h = 0xCBF29CE484222325
    for ch in name.encode():
        h ^= ch
        h = (h * 0x100000001B3) & 0xFFFFFFFFFFFFFFFF
    return h


def _key(seed: int, stream: str) -> np.uint64:
    k = np.array([(int(seed) * 0x9E3779B1 ^ _fnv1a64(stream)) & 0xFFFFFFFFFFFFFFFF],
                 dtype=np.uint64)
    return splitmix64(k)[0]


_BLOCK = 1 << 18   # elements per block: large arrays are generated block by block, in parallel


def _blocks(n: int, fn):
    """Run fn(start, stop) over [0, n) in blocks; several threads for large n (numpy releases the GIL
    inside its elementwise loops).  Every element depends only on its own index, so the result does
    not depend on the block size or the thread count."""
    spans = [(a, min(a + _BLOCK, n)) for a in range(0, n, _BLOCK)]
    if len(spans) <= 2:
        for a, b in spans:
            fn(a, b)
        return
    from concurrent.futures import ThreadPoolExecutor
    import os
    with ThreadPoolExecutor(max_workers=min(16, os.cpu_count() or 1)) as ex:
        list(ex.map(lambda s: fn(*s), spans))


def _uniform_span(key: np.uint64, a: int, b: int) -> np.ndarray:
    idx = np.arange(a, b, dtype=np.uint64)
    with np.errstate(over="ignore"):
        bits = splitmix64(idx + key)
    return (bits >> _U64(11)).astype(np.float64) * (1.0 / 9007199254740992.0)


def uniform(seed: int, stream: str, n: int, lo: float = 0.0, hi: float = 1.0) -> np.ndarray:
    """n float64 uniforms in [lo, hi) for (seed, stream)."""
    key = _key(seed, stream)
    out = np.empty(n, np.float64)

    def fill(a, b):
        out[a:b] = lo + (hi - lo) * _uniform_span(key, a, b)

    _blocks(n, fill)
    return out


def _normal_span(key: np.uint64, a: int, b: int, std: float) -> np.ndarray:
    u = _uniform_span(key, 2 * a, 2 * b)
    r = np.sqrt(-2.0 * np.log1p(-u[0::2]))
    return std * r * np.cos(2.0 * math.pi * u[1::2])


def normal(seed: int, stream: str, n: int, std: float = 1.0) -> np.ndarray:
    """n float64 normals N(0, std^2) for (seed, stream) (Box-Muller, cosine branch): normal j uses
    uniforms 2j and 2j + 1 of the stream."""
    key = _key(seed, stream)
    out = np.empty(n, np.float64)

    def fill(a, b):
        out[a:b] = _normal_span(key, a, b, std)

    _blocks(n, fill)
    return out


# ---------------------------------------------------------------- bf16 bits

def f32_to_bf16(x: np.ndarray) -> np.ndarray:
    """Round float32 to bf16 (round-to-nearest-even); returns uint16 bit patterns."""
    u = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32)
    nan = (u & np.uint32(0x7FFFFFFF)) > np.uint32(0x7F800000)
    r = ((u + np.uint32(0x7FFF) + ((u >> np.uint32(16)) & np.uint32(1))) >> np.uint32(16)).astype(np.uint16)
    if nan.any():
        r = np.where(nan, ((u >> np.uint32(16)) | np.uint32(0x40)).astype(np.uint16), r)
    return r


def bf16_to_f32(h: np.ndarray) -> np.ndarray:
    """Widen bf16 bit patterns (uint16) to float32."""
    return (np.ascontiguousarray(h, dtype=np.uint16).astype(np.uint32) << np.uint32(16)).view(np.float32)


def normal_bf16(seed: int, stream: str, shape, std: float = 1.0) -> np.ndarray:
    """normal(seed, stream, n, std) rounded to f32, then to bf16 bit patterns."""
    n = int(np.prod(shape))
    key = _key(seed, stream)
    out = np.empty(n, np.uint16)

    def fill(a, b):
        out[a:b] = f32_to_bf16(_normal_span(key, a, b, std).astype(np.float32))

    _blocks(n, fill)
    return out.reshape(shape)


# ---------------------------------------------------------------- model config

class GdnConfig:
    """Shapes of one GatedDeltaNet mixer (reference: qwen3_5.rs:506-533)."""

    def __init__(self, hidden=2048, n_k_heads=16, n_v_heads=32, head_k_dim=128,
                 head_v_dim=128, conv_kernel=4, n_layers=30, rms_norm_eps=1e-6):
        self.hidden = hidden
        self.hk = n_k_heads
        self.hv = n_v_heads
        self.dk = head_k_dim
        self.dv = head_v_dim
        self.conv_k = conv_kernel
        self.n_layers = n_layers
        self.eps = rms_norm_eps

    @property
    def conv_dim(self) -> int:          # q + k + v channels (qwen3_5.rs:518)
        return 2 * self.hk * self.dk + self.hv * self.dv

    @property
    def z_dim(self) -> int:
        return self.hv * self.dv

    def as_dict(self):
        return dict(hidden=self.hidden, hk=self.hk, hv=self.hv, dk=self.dk, dv=self.dv,
                    conv_k=self.conv_k, n_layers=self.n_layers, eps=self.eps)


QWEN35_35B_A3B = GdnConfig()


def layer_weights(cfg: GdnConfig, layer: int, with_proj: bool = True) -> dict:
    """Synthetic weights of GDN layer `layer` (seed 1000 + layer).

    Layouts (all row-major):
      conv_w  [D, K] bf16      (reference conv1d weight [D, K, 1])
      A_log   [Hv] f32, dt_bias [Hv] f32
      norm_w  [dv] bf16        (gated RMSNorm gain)
      w_qkv [D, H], w_z [Hv*dv, H], w_b [Hv, H], w_a [Hv, H], w_out [H, Hv*dv] bf16
      pre_w   [H] bf16         (decoder-layer input RMSNorm gain)
    """
    s = 1000 + layer
    D = cfg.conv_dim
    w = {
        "conv_w": normal_bf16(s, "conv_w", (D, cfg.conv_k), 0.02),
        "A_log": uniform(s, "A_log", cfg.hv, 0.0, math.log(16.0)).astype(np.float32),
        "dt_bias": uniform(s, "dt_bias", cfg.hv, -1.0, 1.0).astype(np.float32),
        "norm_w": f32_to_bf16(np.ones(cfg.dv, np.float32)),
        "pre_w": f32_to_bf16(np.ones(cfg.hidden, np.float32)),
    }
    if with_proj:
        H = cfg.hidden
        w["w_qkv"] = normal_bf16(s, "w_qkv", (D, H), 0.02)
        w["w_z"] = normal_bf16(s, "w_z", (cfg.z_dim, H), 0.02)
        w["w_b"] = normal_bf16(s, "w_b", (cfg.hv, H), 0.02)
        w["w_a"] = normal_bf16(s, "w_a", (cfg.hv, H), 0.02)
        w["w_out"] = normal_bf16(s, "w_out", (H, cfg.z_dim), 0.02)
    return w


def quantize_q4(w: np.ndarray, group: int = 64):
    """Affine 4-bit quantization of a bf16 weight [N, K] in groups of `group` columns, in the format of
    MLX's quantize (bits 4; the reference quantizes its projections this way, qwen3_5.rs:929-935):
    weight ~= scale * q + bias with q in 0..15.  Per group: scale = (max - min) / 15 and bias = min,
    both rounded to bf16, then q = clip(round((w - bias) / scale), 0, 15).  (Checkpoints arrive already
    quantized; only the dequantization, scale * q + bias, has to agree with the reference.)

    Returns (w_q [N, K/8] uint32 with column k in bits 4*(k%8) of word k/8, scales, biases [N, K/group]
    bf16)."""
    N, K = w.shape
    assert K % group == 0 and group % 8 == 0
    g = bf16_to_f32(w).astype(np.float64).reshape(N, K // group, group)
    lo, hi = g.min(axis=2), g.max(axis=2)
    scales = f32_to_bf16(((hi - lo) / 15.0).astype(np.float32))
    biases = f32_to_bf16(lo.astype(np.float32))
    s = bf16_to_f32(scales).astype(np.float64)[:, :, None]
    b = bf16_to_f32(biases).astype(np.float64)[:, :, None]
    q = np.where(s > 0, np.rint((g - b) / np.where(s > 0, s, 1.0)), 0.0)
    q = np.clip(q, 0, 15).astype(np.uint32).reshape(N, K // 8, 8)
    w_q = np.zeros((N, K // 8), np.uint32)
    for e in range(8):
        w_q |= q[:, :, e] << np.uint32(4 * e)
    return w_q, scales, biases


def step_inputs(cfg: GdnConfig, n_tokens: int, seed: int = 0, tag: str = "") -> dict:
    """Projection outputs feeding one fused layer step: qkv [N,D], z [N,Hv*dv], ab [N,2Hv] (b then a)."""
    return {
        "qkv": normal_bf16(seed, tag + "qkv", (n_tokens, cfg.conv_dim)),
        "z": normal_bf16(seed, tag + "z", (n_tokens, cfg.z_dim)),
        "ab": normal_bf16(seed, tag + "ab", (n_tokens, 2 * cfg.hv)),
    }


def random_states(cfg: GdnConfig, n_seq: int, seed: int, tag: str = "", scale: float = 0.05):
    """A pre-existing (already prefilled) state per sequence: conv [n,K-1,D] bf16 and rec [n,Hv,dv,dk] f32."""
    conv = normal_bf16(seed, tag + "conv_state", (n_seq, cfg.conv_k - 1, cfg.conv_dim))
    rec = (normal(seed, tag + "rec_state", n_seq * cfg.hv * cfg.dv * cfg.dk) * scale).astype(np.float32)
    return conv, rec.reshape(n_seq, cfg.hv, cfg.dv, cfg.dk)


# ---------------------------------------------------------------- hybrid layers (attention, MoE)

def _rng(seed: int, stream: str) -> np.random.Generator:
    return np.random.default_rng(int(_key(seed, stream)))


def q4_matrix(seed: int, stream: str, rows: int, cols: int, s_scale: float = 0.01) -> dict:
    """A random MLX 4-bit matrix (group 64): uniform codes, scales |N(0, s_scale^2)| + s_scale / 4 and
    biases -8 * scale, both bf16, so dequantised weights centre on 0 with spread ~ 8 * scale."""
    r = _rng(seed, stream)
    q = r.integers(0, 2**32, size=(rows, cols // 8), dtype=np.uint32)
    s = (np.abs(r.standard_normal((rows, cols // 64))) * s_scale + s_scale / 4).astype(np.float32)
    sb = f32_to_bf16(s)
    b = f32_to_bf16((-8.0 * bf16_to_f32(sb)).astype(np.float32))
    return {"q": q, "scales": sb, "biases": b}


def moe_weights(hidden: int, n_experts: int, moe_inter: int, shared_inter: int, seed: int = 0) -> dict:
    """Random-init weights of one SparseMoeBlock (qwen3_5.rs:232-248) in the checkpoint's layout: router and
    shared_expert_gate bf16, experts stacked by rows as 4-bit matrices."""
    return {
        "router": normal_bf16(seed, "moe.router", (n_experts, hidden), 0.02),
        "shared_gate": normal_bf16(seed, "moe.shared_gate", (hidden,), 0.02),
        "gate": q4_matrix(seed, "moe.gate", n_experts * moe_inter, hidden),
        "up": q4_matrix(seed, "moe.up", n_experts * moe_inter, hidden),
        "down": q4_matrix(seed, "moe.down", n_experts * hidden, moe_inter),
        "sh_gate": q4_matrix(seed, "moe.sh_gate", shared_inter, hidden),
        "sh_up": q4_matrix(seed, "moe.sh_up", shared_inter, hidden),
        "sh_down": q4_matrix(seed, "moe.sh_down", hidden, shared_inter),
    }
