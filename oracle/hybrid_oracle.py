"""CPU restatement of the hybrid decoder's attention and MoE layer bodies (TEST INFRASTRUCTURE ONLY).

Only tests/ use this module, as the checker of libgdn_b200.so's gdn_attn_step / gdn_moe_route /
gdn_moe_step.  numpy, vectorised; all bf16 tensors are numpy uint16 bit patterns.

It follows (file:line within the reference project):
  * Qwen35Attention::forward_with_cache   src/models/qwen3_5.rs:377-459
      q_proj output split per head into [queries (hd) | gate (hd)]            :387-391
      q_norm / k_norm: mlx fast::rms_norm                                      :393-404
      partial rope on the first rotary_dim dims, offset = cached length        :410-416
      KV cache concatenation, causal SDPA with scale 1/sqrt(hd)                :419-449
      output gate: attn * sigmoid(gate)                                        :453-456
    with one deliberate difference: each sequence attends only to its own keys.  The reference's
    batched executor zero-pads ragged caches and runs SDPA without a mask
    (src/scheduler/mlx_executor.rs:57-86), which gives padded keys softmax weight; a sequence run
    alone (the reference's own single-sequence path) is what this restates.
  * SparseMoeBlock::forward               src/models/qwen3_5.rs:262-302
      router: softmax(x gate^T), top-k (argpartition), optional renormalisation  :268-284
      SwitchMlp::forward: gather_qmm 4-bit (group 64) gate / up / down          :127-160
      compiled_silu_multiply: silu(a) * b                                      compiled_ops.rs:99-143
      SharedExpert + sigmoid(shared_expert_gate(x)) * shared                     :218-228, :295-300

Rounding points (MLX computes each op in f32 and rounds its output to the array's dtype, bf16):
  rms_norm: bf16(w * bf16(x / sqrt(mean(x^2) + eps)))  (the rule gdn_oracle.c's rms_norm_row states);
  rope: f32 rotation of the bf16 inputs, rounded once; angle = f32(position) * f32(theta^(-i/half));
  SDPA: scores and softmax in f32/f64 from bf16 q, k, v; the output rounded once to bf16;
  sigmoid(gate) bf16, times attention output, bf16;
  router logits bf16; softmax probabilities bf16; renormalised weights bf16(p / bf16(sum p));
  expert projections: the dequantised weight rounded to bf16 (q4_dequant), f32/f64
  accumulation, bf16 output; silu(g) bf16, silu(g) * u bf16; each weighted expert output bf16, their
  sum bf16; sigmoid(shared gate logit) bf16, times the shared expert output bf16; the final add bf16.
Where MLX's kernels accumulate in an order the reference does not fix, this accumulates in f64; the
tests compare with a tolerance for that reason.  MLX itself cannot run here, so these rounding points
are pinned by restatement only.
"""
from __future__ import annotations

import numpy as np

import gdn_oracle as _g


def bf(h: np.ndarray) -> np.ndarray:
    """bf16 bit patterns -> float32 values."""
    return (np.asarray(h, np.uint16).astype(np.uint32) << 16).view(np.float32)


def tobf(x) -> np.ndarray:
    """float32 (or float64, via float32) -> bf16 bit patterns, round to nearest even."""
    x = np.asarray(x)
    if x.dtype == np.float64:
        return _g._f64_to_bf16(x)
    u = np.ascontiguousarray(x, np.float32).view(np.uint32)
    return ((u + np.uint32(0x7FFF) + ((u >> np.uint32(16)) & np.uint32(1))) >> np.uint32(16)).astype(np.uint16)


def rbf(x) -> np.ndarray:
    """float32 values rounded to bf16 precision (round to nearest even), as float32."""
    u = np.ascontiguousarray(x, np.float32).view(np.uint32)
    return ((u + np.uint32(0x7FFF) + ((u >> np.uint32(16)) & np.uint32(1))) & np.uint32(0xFFFF0000)).view(np.float32)


def sigmoid_bf(x: np.ndarray) -> np.ndarray:
    """nn::sigmoid of bf16 values: f32, rounded to bf16 (float32 result)."""
    x = np.asarray(x, np.float32)
    return rbf(np.float32(1.0) / (np.float32(1.0) + np.exp(-x)))


def silu_bf(x: np.ndarray) -> np.ndarray:
    x = np.asarray(x, np.float32)
    return rbf(x * (np.float32(1.0) / (np.float32(1.0) + np.exp(-x))))


def rms_norm_heads(x: np.ndarray, w: np.ndarray, eps: float) -> np.ndarray:
    """mlx fast::rms_norm over the last axis: x bf16 [..., n] -> float32 values of bf16 results."""
    xf = bf(x).astype(np.float64)
    ms = (xf * xf).mean(axis=-1, keepdims=True).astype(np.float32)
    nrm = np.float32(1.0) / np.sqrt(ms + np.float32(eps))
    t = rbf(bf(x) * nrm)
    return rbf(bf(w) * t)


def rope(x: np.ndarray, pos: np.ndarray, rot: int, theta: float) -> np.ndarray:
    """mlx fast::rope, traditional=false (rotate-half pairs (i, i + rot/2)), scale 1, on float32 values of bf16
    inputs x [..., hd] at integer positions pos [...]; returns float32 values of the bf16 results."""
    half = rot // 2
    out = x.astype(np.float32).copy()
    if half == 0:
        return rbf(out)
    inv = (theta ** (-np.arange(half, dtype=np.float64) / half)).astype(np.float32)
    ang = (np.asarray(pos, np.float32)[..., None] * inv).astype(np.float64)
    c, s = np.cos(ang), np.sin(ang)
    x1 = x[..., :half].astype(np.float64)
    x2 = x[..., half:rot].astype(np.float64)
    out[..., :half] = (x1 * c - x2 * s).astype(np.float32)
    out[..., half:rot] = (x1 * s + x2 * c).astype(np.float32)
    return rbf(out)


def attn_step(cfg: dict, q_full, k_in, v_in, q_norm_w, k_norm_w, k_cache, v_cache, slots, cu, positions):
    """One attention layer body over a packed ragged batch (see gdn_hybrid.h, gdn_attn_step).

    cfg: n_heads, n_kv_heads, head_dim, rotary_dim, rope_theta, rms_norm_eps.  k_cache / v_cache bf16
    [n_slots][nkv][max_ctx][hd] are updated in place.  Returns out bf16 [N][nh*hd]."""
    nh, nkv, hd = cfg["n_heads"], cfg["n_kv_heads"], cfg["head_dim"]
    rot, theta, eps = cfg["rotary_dim"], cfg["rope_theta"], cfg["rms_norm_eps"]
    G = nh // nkv
    N = q_full.shape[0]
    qf = np.asarray(q_full, np.uint16).reshape(N, nh, 2 * hd)
    out = np.zeros((N, nh * hd), np.uint16)
    scale = np.float32(1.0) / np.sqrt(np.float32(hd))
    for i in range(len(slots)):
        b, e = int(cu[i]), int(cu[i + 1])
        if e == b:
            continue
        s, p0 = int(slots[i]), int(positions[i])
        pos = p0 + np.arange(e - b)
        q = rope(rms_norm_heads(qf[b:e, :, :hd], q_norm_w, eps), pos[:, None], rot, theta)     # [T, nh, hd]
        kk = np.asarray(k_in[b:e], np.uint16).reshape(e - b, nkv, hd)
        k = rope(rms_norm_heads(kk, k_norm_w, eps), pos[:, None], rot, theta)                   # [T, nkv, hd]
        v = np.asarray(v_in[b:e], np.uint16).reshape(e - b, nkv, hd)
        k_cache[s, :, p0:p0 + (e - b)] = tobf(k).transpose(1, 0, 2)
        v_cache[s, :, p0:p0 + (e - b)] = v.transpose(1, 0, 2)
        K = bf(k_cache[s, :, :p0 + (e - b)]).astype(np.float64)                                # [nkv, L, hd]
        V = bf(v_cache[s, :, :p0 + (e - b)]).astype(np.float64)
        L = p0 + (e - b)
        gate = bf(qf[b:e, :, hd:])
        for hh in range(nh):
            kv = hh // G
            sc = (q[:, hh].astype(np.float64) * np.float64(scale)) @ K[kv].T                  # [T, L]
            mask = np.arange(L)[None, :] > pos[:, None]
            sc[mask] = -np.inf
            sc -= sc.max(axis=1, keepdims=True)
            pr = np.exp(sc)
            pr /= pr.sum(axis=1, keepdims=True)
            o = rbf((pr @ V[kv]).astype(np.float32))
            out[b:e, hh * hd:(hh + 1) * hd] = tobf(o * sigmoid_bf(gate[:, hh]))
    return out


# ------------------------------------------------------------------ MoE

def moe_logits(x, router):
    """Router logits bf16 [N][E] = bf16(x router^T) (f64 accumulation)."""
    return _g._f64_to_bf16(bf(x).astype(np.float64) @ bf(router).astype(np.float64).T)


def moe_route(logits, top_k: int, norm: bool):
    """softmax (f32, probabilities rounded to bf16), the top_k experts by probability (descending, lower
    index first among equal probabilities), weights renormalised in bf16 when `norm`.
    Returns (ids int32 [N][k], weights bf16 [N][k], probabilities float32 [N][E])."""
    lf = bf(logits).astype(np.float64)
    ex = np.exp(lf - lf.max(axis=1, keepdims=True))
    p = rbf((ex / ex.sum(axis=1, keepdims=True)).astype(np.float32))
    N, E = p.shape
    order = np.lexsort((np.broadcast_to(np.arange(E), (N, E)), -p), axis=1)   # by -p, then index
    ids = order[:, :top_k].astype(np.int32)
    w = np.take_along_axis(p, ids, axis=1)
    if norm:
        den = rbf(w.astype(np.float32).sum(axis=1, dtype=np.float32, keepdims=True))
        w = w / den
    return ids, tobf(w.astype(np.float32)), p


def q4_dequant(m: dict, rows: slice) -> np.ndarray:
    """Rows of an MLX 4-bit matrix dequantised to bf16 (the rule of gdn_oracle.q4_dequantize): scale * q + bias
    rounded once.  In f32, where the product of a bf16 scale and a 4-bit code and its sum with a bf16 bias
    of the same scale are exact, so this equals the f64 form bit for bit (a CPU test checks it)."""
    q = np.asarray(m["q"][rows], np.uint32)
    R, W = q.shape
    shifts = (np.arange(8, dtype=np.uint32) * 4)[None, None, :]
    codes = ((q[:, :, None] >> shifts) & np.uint32(0xF)).astype(np.float32).reshape(R, W // 8, 64)
    sc = bf(m["scales"][rows])[:, :, None]
    bi = bf(m["biases"][rows])[:, :, None]
    return tobf((codes * sc + bi).reshape(R, W * 8))


def _q4_f64(m: dict, rows: slice) -> np.ndarray:
    q = np.asarray(m["q"][rows], np.uint32)
    R, W = q.shape
    shifts = (np.arange(8, dtype=np.uint32) * 4)[None, None, :]
    codes = ((q[:, :, None] >> shifts) & np.uint32(0xF)).astype(np.float32).reshape(R, W // 8, 64)
    return rbf(codes * bf(m["scales"][rows])[:, :, None] + bf(m["biases"][rows])[:, :, None]).reshape(
        R, W * 8).astype(np.float64)


def _mlp(x_f64, gq: dict, uq: dict, dq: dict, erow_g: slice, erow_d: slice):
    """down(silu(gate x) * up x) for token rows x (float64 values of bf16), one expert's rows."""
    Wg = _q4_f64(gq, erow_g)   # q4_dequant's values, as f64
    Wu = _q4_f64(uq, erow_g)
    Wd = _q4_f64(dq, erow_d)
    g = bf(_g._f64_to_bf16(x_f64 @ Wg.T))
    u = bf(_g._f64_to_bf16(x_f64 @ Wu.T))
    h = rbf(silu_bf(g) * u)
    return bf(_g._f64_to_bf16(h.astype(np.float64) @ Wd.T))


def moe_step(cfg: dict, w: dict, x, ids=None, weights=None):
    """The MoE block (see gdn_hybrid.h, gdn_moe_step).  cfg: hidden, n_experts, top_k, moe_inter,
    shared_inter, norm_topk_prob.  w: router bf16 [E][H]; gate / up / down / sh_gate / sh_up / sh_down
    as dicts of q (uint32), scales, biases (bf16) with experts stacked by rows; shared_gate bf16 [H].
    ids / weights: a routing to use instead of the router's."""
    H, E, K, I = cfg["hidden"], cfg["n_experts"], cfg["top_k"], cfg["moe_inter"]
    x = np.asarray(x, np.uint16)
    N = x.shape[0]
    if ids is None:
        ids, weights, _ = moe_route(moe_logits(x, w["router"]), K, bool(cfg["norm_topk_prob"]))
    xf = bf(x).astype(np.float64)
    wf = bf(weights)
    contrib = np.zeros((N, K, H), np.float32)   # bf16(y_j * w_j) per (token, k)
    for e in np.unique(ids):
        tok, j = np.nonzero(ids == e)
        y = _mlp(xf[tok], w["gate"], w["up"], w["down"], slice(e * I, (e + 1) * I), slice(e * H, (e + 1) * H))
        contrib[tok, j] = rbf(y * wf[tok, j][:, None])
    acc = np.zeros((N, H), np.float32)
    for j in range(K):   # summed over k in order, f32
        acc = (acc + contrib[:, j]).astype(np.float32)
    moe = rbf(acc)
    Hs = cfg["shared_inter"]
    ys = _mlp(xf, w["sh_gate"], w["sh_up"], w["sh_down"], slice(0, Hs), slice(0, H))
    sg = bf(_g._f64_to_bf16(xf @ bf(w["shared_gate"]).astype(np.float64)))
    shg = rbf(sigmoid_bf(sg)[:, None] * ys)
    return tobf(moe + shg)

