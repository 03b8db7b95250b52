"""ctypes front end of the CPU oracle (TEST INFRASTRUCTURE ONLY).

Only tests/, __graft_entry__.smoke() and bench.py's cpu_baseline / --impl
reference legs use this module, and only as the checker or the timed CPU
baseline.  It wraps:

  * oracle/_build/libgdn_oracle.so  -- C restatement of the reference layer
    (see gdn_oracle.c for the reference file:line it follows);
  * oracle/_ref/libgdn_metal_ref.so -- the reference's own Metal kernel body
    (metal_gdn.rs:10-67) compiled for the CPU, when it has been built;
  * f64 numpy restatements used as an independent cross-check of the
    recurrence algebra (no bf16 rounding inside, so they bound rather than
    match the oracle).

All bf16 tensors are numpy uint16 bit patterns.
"""
from __future__ import annotations

import ctypes as C
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
ORACLE_SO = HERE / "_build" / "libgdn_oracle.so"
REF_SO = HERE / "_ref" / "libgdn_metal_ref.so"

_u16p = np.ctypeslib.ndpointer(np.uint16, flags="C_CONTIGUOUS")
_f32p = np.ctypeslib.ndpointer(np.float32, flags="C_CONTIGUOUS")
_i32p = np.ctypeslib.ndpointer(np.int32, flags="C_CONTIGUOUS")


class OrcCfg(C.Structure):
    _fields_ = [("hidden", C.c_int32), ("hk", C.c_int32), ("hv", C.c_int32), ("dk", C.c_int32),
                ("dv", C.c_int32), ("conv_k", C.c_int32), ("eps", C.c_float)]


class OrcLayerW(C.Structure):
    _fields_ = [("conv_w", C.c_void_p), ("A_log", C.c_void_p), ("dt_bias", C.c_void_p), ("norm_w", C.c_void_p),
                ("dt_bias_bf16", C.c_int32)]


class OrcMixerW(C.Structure):
    _fields_ = [("core", OrcLayerW), ("w_qkv", C.c_void_p), ("w_z", C.c_void_p), ("w_b", C.c_void_p),
                ("w_a", C.c_void_p), ("w_out", C.c_void_p), ("pre_w", C.c_void_p)]


_lib = None
_ref = None


def lib():
    global _lib
    if _lib is None:
        if not ORACLE_SO.exists():
            raise FileNotFoundError(f"{ORACLE_SO} missing: run oracle/build.py (or __graft_entry__.build())")
        L = C.CDLL(str(ORACLE_SO))
        L.orc_recurrence.argtypes = [_u16p, _u16p, _u16p, _f32p, _u16p, _f32p, C.c_int32, C.c_int32, C.c_int32,
                                     C.c_int32, C.c_int32, C.c_int32, _u16p]
        L.orc_recurrence.restype = C.c_int
        L.orc_recurrence_packed.argtypes = [_u16p, _u16p, _u16p, _f32p, _u16p, _f32p, _i32p, C.c_int32, C.c_int32,
                                            C.c_int32, C.c_int32, C.c_int32, _u16p]
        L.orc_recurrence_packed.restype = C.c_int
        L.orc_gates.argtypes = [_u16p, C.c_int64, C.c_int64, C.c_int32, _f32p, _f32p, C.c_int32, _f32p, _u16p]
        L.orc_gates.restype = None
        L.orc_rms_norm.argtypes = [_u16p, _u16p, C.c_int64, C.c_int32, C.c_float, _u16p]
        L.orc_rms_norm.restype = None
        L.orc_linear.argtypes = [_u16p, _u16p, C.c_int64, C.c_int32, C.c_int32, _u16p]
        L.orc_linear.restype = None
        L.orc_layer_step.argtypes = [C.POINTER(OrcCfg), C.POINTER(OrcLayerW), C.c_void_p, C.c_int64, C.c_void_p,
                                     C.c_int64, C.c_void_p, C.c_int64, _u16p, _f32p, _i32p, C.c_int32, _u16p,
                                     C.c_void_p]
        L.orc_layer_step.restype = C.c_int
        L.orc_mixer_step.argtypes = [C.POINTER(OrcCfg), C.POINTER(OrcMixerW), _u16p, _u16p, _f32p, _i32p,
                                     C.c_int32, _u16p]
        L.orc_mixer_step.restype = C.c_int
        L.orc_stack_step.argtypes = [C.POINTER(OrcCfg), C.POINTER(OrcMixerW), C.c_int32, _u16p, _u16p, _f32p,
                                     _i32p, C.c_int32]
        L.orc_stack_step.restype = C.c_int
        L.orc_conv.argtypes = [C.POINTER(OrcCfg), _u16p, C.c_int64, C.c_int32, _u16p, _u16p, _u16p]
        L.orc_conv.restype = C.c_int
        L.orc_set_linear_order.argtypes = [C.c_int]
        L.orc_set_linear_order.restype = None
        L.orc_num_threads.restype = C.c_int
        L.orc_set_num_threads.argtypes = [C.c_int]
        _lib = L
    return _lib


def ref_lib():
    """The CPU-compiled reference Metal kernel, or None when it was not built here."""
    global _ref
    if _ref is None and REF_SO.exists():
        L = C.CDLL(str(REF_SO))
        L.mref_gated_delta_kernel.argtypes = [_u16p, _u16p, _u16p, _f32p, _u16p, _f32p, C.c_int, C.c_int, C.c_int,
                                              C.c_int, C.c_int, C.c_int, _u16p, _f32p]
        L.mref_gated_delta_kernel.restype = C.c_int
        _ref = L
    return _ref


def _c(a, dt):
    return np.ascontiguousarray(a, dtype=dt)


def cfg_struct(cfg) -> OrcCfg:
    return OrcCfg(cfg.hidden, cfg.hk, cfg.hv, cfg.dk, cfg.dv, cfg.conv_k, cfg.eps)


def set_linear_order(order: int):
    """Accumulation order of orc_linear: 0 sequential (default); 1 32 interleaved partial sums + tree;
    2 blocks of 16 accumulated in order; 3 reverse sequential."""
    lib().orc_set_linear_order(int(order))


def set_threads(n: int):
    lib().orc_set_num_threads(int(n))


def num_threads() -> int:
    return int(lib().orc_num_threads())


# ------------------------------------------------------------------ wrappers

def recurrence(q, k, v, g, beta, state, T, B, hk, hv, dk, dv):
    """Reference-shaped recurrence (metal_gdn.rs:170): returns (y, new_state); inputs untouched."""
    st = _c(state, np.float32).copy()
    y = np.zeros((B, T, hv, dv), np.uint16)
    rc = lib().orc_recurrence(_c(q, np.uint16), _c(k, np.uint16), _c(v, np.uint16), _c(g, np.float32),
                              _c(beta, np.uint16), st, T, B, hk, hv, dk, dv, y)
    if rc:
        raise ValueError(f"orc_recurrence rc={rc}")
    return y, st


def recurrence_packed(q, k, v, g, beta, states, cu, hk, hv, dk, dv):
    """Packed ragged recurrence over dense per-sequence states; returns (y, new_states)."""
    cu = _c(cu, np.int32)
    st = _c(states, np.float32).copy()
    N = int(cu[-1])
    y = np.zeros((N, hv, dv), np.uint16)
    rc = lib().orc_recurrence_packed(_c(q, np.uint16), _c(k, np.uint16), _c(v, np.uint16), _c(g, np.float32),
                                     _c(beta, np.uint16), st, cu, len(cu) - 1, hk, hv, dk, dv, y)
    if rc:
        raise ValueError(f"orc_recurrence_packed rc={rc}")
    return y, st


def ref_recurrence(q, k, v, g, beta, state, T, B, hk, hv, dk, dv):
    """The reference Metal kernel compiled for the CPU; None when unavailable."""
    L = ref_lib()
    if L is None:
        return None
    y = np.zeros((B, T, hv, dv), np.uint16)
    st_out = np.zeros((B, hv, dv, dk), np.float32)
    rc = L.mref_gated_delta_kernel(_c(q, np.uint16), _c(k, np.uint16), _c(v, np.uint16), _c(g, np.float32),
                                   _c(beta, np.uint16), _c(state, np.float32), T, B, hk, hv, dk, dv, y, st_out)
    if rc:
        raise ValueError(f"reference kernel has no instantiation for hk={hk} hv={hv} dk={dk} dv={dv}")
    return y, st_out


def gates(ab, A_log, dt_bias, hv, dt_bias_bf16=False):
    """compiled_beta_g: (g f32, beta bf16).  dt_bias_bf16: the checkpoint stores dt_bias in bf16 (passed
    widened to f32), so a + dt_bias and its exp round to bf16 as MLX computes them."""
    ab = _c(ab, np.uint16)
    n = ab.shape[0]
    g = np.zeros((n, hv), np.float32)
    beta = np.zeros((n, hv), np.uint16)
    lib().orc_gates(ab, ab.shape[1], n, hv, _c(A_log, np.float32), _c(dt_bias, np.float32),
                    1 if dt_bias_bf16 else 0, g, beta)
    return g, beta


def rms_norm(x, w, eps):
    x = _c(x, np.uint16)
    out = np.zeros_like(x)
    n = x.shape[-1]
    lib().orc_rms_norm(x, _c(w, np.uint16), x.size // n, n, eps, out)
    return out


def linear(x, w):
    x = _c(x, np.uint16)
    w = _c(w, np.uint16)
    M, K = x.shape
    N = w.shape[0]
    out = np.zeros((M, N), np.uint16)
    lib().orc_linear(x, w, M, N, K, out)
    return out


def _f64_to_bf16(x):
    """Round float64 to bf16 once (round-to-nearest-even): via float32 rounded to odd, which keeps the
    information a second rounding to bf16 needs."""
    x = np.asarray(x, np.float64)
    t = x.astype(np.float32)
    over = np.abs(t.astype(np.float64)) > np.abs(x)
    t = np.where(over, np.nextafter(t, np.float32(0)), t).astype(np.float32)
    inexact = t.astype(np.float64) != x
    u = t.view(np.uint32) | inexact.astype(np.uint32)
    u32 = u.astype(np.uint32)
    return ((u32 + np.uint32(0x7FFF) + ((u32 >> np.uint32(16)) & np.uint32(1))) >> np.uint32(16)).astype(np.uint16)


def q4_dequantize(w_q, scales, biases, group: int = 64):
    """MLX affine 4-bit dequantization (bits 4, groups of `group` columns; mlx quantized_matmul with
    transpose, called for the quantized projections at qwen3_5.rs:572-586, :668): column k of row n is
    scale[n][k/group] * q + bias[n][k/group], q = bits 4*(k%8) of word k/8, rounded once to the
    activation type (bf16), as MLX's quantized matmul tile loader writes it.  Returns bf16 [N, K]."""
    w_q = np.asarray(w_q, np.uint32)
    N, K = w_q.shape[0], w_q.shape[1] * 8
    shifts = (np.arange(8, dtype=np.uint32) * 4)[None, None, :]
    q = ((w_q[:, :, None] >> shifts) & np.uint32(0xF)).reshape(N, K).astype(np.float64)
    s = np.repeat((np.asarray(scales, np.uint16).astype(np.uint32) << 16).view(np.float32).astype(np.float64),
                  group, axis=1)
    b = np.repeat((np.asarray(biases, np.uint16).astype(np.uint32) << 16).view(np.float32).astype(np.float64),
                  group, axis=1)
    return _f64_to_bf16(s * q + b)


def q4_linear(x, w_q, scales, biases):
    """The 4-bit projection: bf16(x @ dequant(w)^T) with f32 accumulation (linear() on the
    dequantized weight)."""
    return linear(x, q4_dequantize(w_q, scales, biases))


def conv(cfg, x, conv_state, conv_w):
    """Causal conv + SiLU over one sequence x [T, >=D]; returns (out [T, D], new conv state)."""
    x = _c(x, np.uint16)
    cs = _c(conv_state, np.uint16).copy()
    out = np.zeros((x.shape[0], cfg.conv_dim), np.uint16)
    c = cfg_struct(cfg)
    lib().orc_conv(C.byref(c), x, x.shape[1], x.shape[0], cs, _c(conv_w, np.uint16), out)
    return out, cs


def _layer_w(w):
    keep = {k: _c(w[k], np.uint16 if k in ("conv_w", "norm_w") else np.float32)
            for k in ("conv_w", "A_log", "dt_bias", "norm_w")}
    s = OrcLayerW(keep["conv_w"].ctypes.data, keep["A_log"].ctypes.data, keep["dt_bias"].ctypes.data,
                  keep["norm_w"].ctypes.data, 1 if w.get("dt_bias_bf16", False) else 0)
    return s, keep


def layer_step(cfg, w, qkv, z, ab, conv_state, rec_state, cu, want_y=False):
    """One fused layer step over a packed batch; states are dense per sequence.

    Returns (out [N, Hv*dv], conv_state', rec_state', y or None).
    """
    cu = _c(cu, np.int32)
    n_seq = len(cu) - 1
    N = int(cu[-1])
    qkv = _c(qkv, np.uint16)
    z = _c(z, np.uint16)
    ab = _c(ab, np.uint16)
    cs = _c(conv_state, np.uint16).copy()
    rs = _c(rec_state, np.float32).copy()
    out = np.zeros((N, cfg.hv * cfg.dv), np.uint16)
    y = np.zeros((N, cfg.hv * cfg.dv), np.uint16) if want_y else None
    ws, keep = _layer_w(w)
    c = cfg_struct(cfg)
    rc = lib().orc_layer_step(C.byref(c), C.byref(ws), qkv.ctypes.data, qkv.shape[1], z.ctypes.data, z.shape[1],
                              ab.ctypes.data, ab.shape[1], cs, rs, cu, n_seq, out,
                              y.ctypes.data if y is not None else None)
    del keep
    if rc:
        raise ValueError(f"orc_layer_step rc={rc}")
    return out, cs, rs, y


def _mixer_w(w):
    core, keep = _layer_w(w)
    for k in ("w_qkv", "w_z", "w_b", "w_a", "w_out", "pre_w"):
        keep[k] = _c(w[k], np.uint16)
    s = OrcMixerW(core, keep["w_qkv"].ctypes.data, keep["w_z"].ctypes.data, keep["w_b"].ctypes.data,
                  keep["w_a"].ctypes.data, keep["w_out"].ctypes.data, keep["pre_w"].ctypes.data)
    return s, keep


def mixer_step(cfg, w, x, conv_state, rec_state, cu):
    cu = _c(cu, np.int32)
    cs = _c(conv_state, np.uint16).copy()
    rs = _c(rec_state, np.float32).copy()
    N = int(cu[-1])
    out = np.zeros((N, cfg.hidden), np.uint16)
    ws, keep = _mixer_w(w)
    c = cfg_struct(cfg)
    rc = lib().orc_mixer_step(C.byref(c), C.byref(ws), _c(x, np.uint16), cs, rs, cu, len(cu) - 1, out)
    del keep
    if rc:
        raise ValueError(f"orc_mixer_step rc={rc}")
    return out, cs, rs


def stack_step(cfg, ws, h, conv_state, rec_state, cu):
    """h <- h + mixer_l(rms_norm(h)) over len(ws) layers; states [L][n_seq][...]."""
    cu = _c(cu, np.int32)
    h = _c(h, np.uint16).copy()
    cs = _c(conv_state, np.uint16).copy()
    rs = _c(rec_state, np.float32).copy()
    arr = (OrcMixerW * len(ws))()
    keeps = []
    for i, w in enumerate(ws):
        s, keep = _mixer_w(w)
        arr[i] = s
        keeps.append(keep)
    c = cfg_struct(cfg)
    rc = lib().orc_stack_step(C.byref(c), arr, len(ws), h, cs, rs, cu, len(cu) - 1)
    del keeps
    if rc:
        raise ValueError(f"orc_stack_step rc={rc}")
    return h, cs, rs


# ------------------------------------------------------- f64 cross-checks

def f64_recurrence(q, k, v, g, beta, state, hk, hv):
    """Plain float64 gated delta rule on dense [T, heads, d] inputs of ONE sequence.

    q, k, v, beta given as float arrays (already widened); state [hv, dv, dk].
    S_t = g S + beta (v - g S k) k^T ; y_t = S_t q.
    """
    S = state.astype(np.float64).copy()
    T = q.shape[0]
    dv = S.shape[1]
    y = np.zeros((T, hv, dv))
    r = hv // hk
    for t in range(T):
        for h in range(hv):
            kk = k[t, h // r].astype(np.float64)
            qq = q[t, h // r].astype(np.float64)
            S[h] *= g[t, h]
            kv = S[h] @ kk
            delta = (v[t, h].astype(np.float64) - kv) * beta[t, h]
            S[h] += np.outer(delta, kk)
            y[t, h] = S[h] @ qq
    return y, S
