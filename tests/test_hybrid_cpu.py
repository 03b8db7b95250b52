"""CPU tests of the attention / MoE layer bodies: the oracle's own properties and pins, and the C ABI's host-side
argument checks (no GPU work is issued: every call here fails its checks before touching the device)."""
from __future__ import annotations

import ctypes as C
import importlib

import numpy as np
import pytest


@pytest.fixture(scope="module")
def H():
    import __graft_entry__ as ge
    ge.load_oracle()
    return importlib.import_module("hybrid_oracle")


@pytest.fixture(scope="module")
def hy(pkg):
    return importlib.import_module("qwen_mlx_b200.hybrid")


# ------------------------------------------------------------------ oracle pins and properties

def test_q4_dequant_matches_projection_oracle(H, synth, oracle):
    """The experts' dequantisation is the projections' (gdn_oracle.q4_dequantize), bit for bit."""
    m = synth.q4_matrix(3, "pin", 128, 512)
    assert np.array_equal(H.q4_dequant(m, slice(0, 128)), oracle.q4_dequantize(m["q"], m["scales"], m["biases"]))


def test_rope_depends_on_relative_position(H):
    """<rope(q, m), rope(k, n)> depends on m - n only (up to the bf16 rounding of the rotated vectors)."""
    rng = np.random.default_rng(0)
    q = rng.standard_normal(256).astype(np.float32)
    k = rng.standard_normal(256).astype(np.float32)
    dots = [float(H.rope(q[None], np.array([m]), 64, 1e7)[0] @ H.rope(k[None], np.array([m - 7]), 64, 1e7)[0])
            for m in (7, 100, 1000, 4000)]
    assert np.ptp(dots) < 2e-2 * abs(dots[0]) + 0.05
    # dims past rotary_dim are untouched (only rounded)
    r = H.rope(q[None], np.array([123]), 64, 1e7)[0]
    assert np.array_equal(r[64:], H.rbf(q[64:]))


def test_attn_oracle_masks_other_keys(H, synth):
    """A token's output ignores cache rows past its position and every other slot's rows."""
    cfg = dict(n_heads=4, n_kv_heads=2, head_dim=64, rotary_dim=16, rope_theta=1e4, rms_norm_eps=1e-6)
    rng = np.random.default_rng(1)
    bfr = lambda shape: synth.f32_to_bf16(rng.standard_normal(shape).astype(np.float32))  # noqa: E731
    qf, kin, vin = bfr((3, 4 * 128)), bfr((3, 2 * 64)), bfr((3, 2 * 64))
    qn = kn = synth.f32_to_bf16(np.ones(64, np.float32))
    kc, vc = bfr((2, 2, 32, 64)), bfr((2, 2, 32, 64))
    out1 = H.attn_step(cfg, qf, kin, vin, qn, kn, kc.copy(), vc.copy(), [1], [0, 3], [5])
    kc2, vc2 = kc.copy(), vc.copy()
    kc2[1, :, 8:] = bfr((2, 24, 64))   # rows past the last token's position (7)
    vc2[1, :, 8:] = bfr((2, 24, 64))
    kc2[0], vc2[0] = bfr((2, 32, 64)), bfr((2, 32, 64))
    out2 = H.attn_step(cfg, qf, kin, vin, qn, kn, kc2, vc2, [1], [0, 3], [5])
    assert np.array_equal(out1, out2)


def test_moe_route_ties_and_renormalisation(H, synth):
    logits = synth.f32_to_bf16(np.array([[1.0, 3.0, 3.0, 2.0, 3.0, -1.0]], np.float32))
    ids, w, p = H.moe_route(logits, 3, True)
    assert ids.tolist() == [[1, 2, 4]]   # equal probabilities: lower index first
    assert abs(float(H.bf(w).sum()) - 1.0) < 1e-2
    ids2, w2, _ = H.moe_route(logits, 3, False)
    assert np.array_equal(H.bf(w2), p[0, [1, 2, 4]][None])


# ------------------------------------------------------------------ ABI host checks

def _acfg(hy, **kw):
    return hy.AttnConfig(**kw).c()


def test_attn_workspace_query(abi, hy):
    L = abi.lib()
    out = C.c_int64(0)
    assert L.gdn_attn_workspace_bytes(C.byref(_acfg(hy)), 8, 4096, C.byref(out)) == abi.GDN_OK
    # 8 decode tokens, 16 heads of 256: per-(token, head) partials of up to 16 key splits dominate
    assert out.value >= 8 * 16 * 16 * 256 * 4
    assert L.gdn_attn_workspace_bytes(C.byref(_acfg(hy, head_dim=96)), 8, 64, C.byref(out)) == abi.GDN_E_UNSUPPORTED
    assert L.gdn_attn_workspace_bytes(C.byref(_acfg(hy, n_heads=6, n_kv_heads=4)), 8, 64, C.byref(out)) == \
        abi.GDN_E_INVALID
    assert L.gdn_attn_workspace_bytes(C.byref(_acfg(hy, rotary_dim=63)), 8, 64, C.byref(out)) == abi.GDN_E_INVALID


@pytest.mark.parametrize("slots,lens,positions,code", [
    ([1, 1], [1, 1], [0, 0], 3),        # slot used twice
    ([4], [1], [0], 3),                 # slot out of range (4 slots)
    ([0, 1], [1, 2], [0, 15], 1),       # position + tokens past max_ctx (16)
    ([0], [1], [-1], 1),                # negative position
])
def test_attn_step_rejects_bad_tables(abi, hy, slots, lens, positions, code):
    cfg = _acfg(hy, max_ctx=16)
    s = np.asarray(slots, np.int32)
    cu = np.concatenate([[0], np.cumsum(lens)]).astype(np.int32)
    pos = np.asarray(positions, np.int32)
    fake = C.c_void_p(256)   # device pointers are never touched on a failing call
    rc = abi.lib().gdn_attn_step(C.byref(cfg), fake, fake, fake, fake, fake, fake, fake, 4,
                                 s.ctypes.data_as(C.c_void_p), cu.ctypes.data_as(C.c_void_p),
                                 pos.ctypes.data_as(C.c_void_p), len(s), int(cu[-1]), fake, fake, 1 << 30, None)
    assert rc == code, abi.last_error()
    assert abi.last_error()


def test_attn_step_bad_seqlens(abi, hy):
    cfg = _acfg(hy, max_ctx=16)
    s = np.asarray([0, 1], np.int32)
    cu = np.asarray([0, 2, 1], np.int32)
    pos = np.zeros(2, np.int32)
    fake = C.c_void_p(256)
    rc = abi.lib().gdn_attn_step(C.byref(cfg), fake, fake, fake, fake, fake, fake, fake, 4,
                                 s.ctypes.data_as(C.c_void_p), cu.ctypes.data_as(C.c_void_p),
                                 pos.ctypes.data_as(C.c_void_p), 2, 1, fake, fake, 1 << 30, None)
    assert rc == abi.GDN_E_BAD_SEQLENS


def test_moe_workspace_and_checks(abi, hy):
    L = abi.lib()
    out = C.c_int64(0)
    cfg = hy.MoeConfig()
    assert L.gdn_moe_workspace_bytes(C.byref(cfg.c()), 8, C.byref(out)) == abi.GDN_OK
    assert out.value >= 8 * 9 * (512 + 2048) * 2   # h and y rows of every (token, expert) pair
    bad = hy.MoeConfig(hidden=2000).c()
    assert L.gdn_moe_workspace_bytes(C.byref(bad), 8, C.byref(out)) == abi.GDN_E_UNSUPPORTED
    bad = hy.MoeConfig(top_k=17).c()
    assert L.gdn_moe_workspace_bytes(C.byref(bad), 8, C.byref(out)) == abi.GDN_E_UNSUPPORTED
    # routing given half-way: rejected before any launch
    fake = C.c_void_p(256)
    q = abi.GdnQ4MatrixC(fake, fake, fake)
    w = abi.GdnMoeWeightsC(fake, q, q, q, q, q, q, fake)
    rc = L.gdn_moe_step(C.byref(cfg.c()), C.byref(w), fake, 4, fake, None, fake, fake, 1 << 30, None)
    assert rc == abi.GDN_E_INVALID
    rc = L.gdn_moe_step(C.byref(cfg.c()), C.byref(w), fake, 4, None, None, fake, fake, 16, None)
    assert rc == abi.GDN_E_INVALID and "workspace" in abi.last_error()


# ------------------------------------------------------------------ independent f64 cross-checks of the oracle

def _f64_attention(H, cfg, qf, kin, vin, qn, kn, kc, vc, slots, cu, positions):
    """Token by token, in f64 without any bf16 rounding: the same layer written a second way (explicit loops,
    rotation by angle pairs, a plain softmax), to bound the rounded oracle."""
    nh, nkv, hd, rot = cfg["n_heads"], cfg["n_kv_heads"], cfg["head_dim"], cfg["rotary_dim"]
    th, eps = cfg["rope_theta"], cfg["rms_norm_eps"]
    G, half = nh // nkv, rot // 2
    qf = H.bf(qf).astype(np.float64).reshape(len(qf), nh, 2 * hd)
    kin = H.bf(kin).astype(np.float64).reshape(len(kin), nkv, hd)
    vin = H.bf(vin).astype(np.float64).reshape(len(vin), nkv, hd)
    Kc, Vc = H.bf(kc).astype(np.float64), H.bf(vc).astype(np.float64)
    qn, kn = H.bf(qn).astype(np.float64), H.bf(kn).astype(np.float64)

    def norm_rope(x, g, p):
        y = x / np.sqrt(np.mean(x * x) + eps) * g
        out = y.copy()
        for i in range(half):
            a = p * th ** (-i / half)
            out[i] = y[i] * np.cos(a) - y[i + half] * np.sin(a)
            out[i + half] = y[i] * np.sin(a) + y[i + half] * np.cos(a)
        return out

    out = np.zeros((len(qf), nh * hd))
    for s_i, s in enumerate(slots):
        for t in range(cu[s_i], cu[s_i + 1]):
            p = positions[s_i] + (t - cu[s_i])
            for kv in range(nkv):
                Kc[s, kv, p] = norm_rope(kin[t, kv], kn, p)
                Vc[s, kv, p] = vin[t, kv]
        for t in range(cu[s_i], cu[s_i + 1]):
            p = positions[s_i] + (t - cu[s_i])
            for h in range(nh):
                q = norm_rope(qf[t, h, :hd], qn, p)
                sc = np.array([q @ Kc[s, h // G, j] for j in range(p + 1)]) / np.sqrt(hd)
                w = np.exp(sc - sc.max())
                o = (w / w.sum()) @ Vc[s, h // G, :p + 1]
                out[t, h * hd:(h + 1) * hd] = o / (1.0 + np.exp(-qf[t, h, hd:]))
    return out


def test_attention_oracle_bounded_by_f64_restatement(H, synth):
    cfg = dict(n_heads=4, n_kv_heads=2, head_dim=64, rotary_dim=16, rope_theta=1e4, rms_norm_eps=1e-6)
    rng = np.random.default_rng(7)
    bfr = lambda shape: synth.f32_to_bf16(rng.standard_normal(shape).astype(np.float32))  # noqa: E731
    slots, lens, positions = [1, 0], [3, 1], [2, 5]
    cu = np.concatenate([[0], np.cumsum(lens)]).astype(np.int32)
    qf, kin, vin = bfr((4, 4 * 128)), bfr((4, 2 * 64)), bfr((4, 2 * 64))
    qn = synth.f32_to_bf16((1 + 0.1 * rng.standard_normal(64)).astype(np.float32))
    kn = synth.f32_to_bf16((1 + 0.1 * rng.standard_normal(64)).astype(np.float32))
    kc, vc = bfr((2, 2, 8, 64)), bfr((2, 2, 8, 64))
    got = H.bf(H.attn_step(cfg, qf, kin, vin, qn, kn, kc.copy(), vc.copy(), slots, cu, positions))
    ref = _f64_attention(H, cfg, qf, kin, vin, qn, kn, kc, vc, slots, cu, positions)
    err = np.linalg.norm(got - ref) / np.linalg.norm(ref)
    assert err < 1e-2   # bf16 roundings of q, k, the SDPA output, the gate and the product


def test_moe_oracle_bounded_by_per_pair_restatement(H, synth):
    """The oracle groups pairs by expert; this runs every (token, k) pair on its own in f64 without bf16
    rounding (other than the dequantised weights), then weights, sums and adds the gated shared expert."""
    cfg = dict(hidden=128, n_experts=6, top_k=3, moe_inter=64, shared_inter=64, norm_topk_prob=True)
    w = synth.moe_weights(128, 6, 64, 64, seed=11)
    x = synth.normal_bf16(11, "pp.x", (5, 128))
    got = H.bf(H.moe_step(cfg, w, x))
    xf = H.bf(x).astype(np.float64)
    logits = xf @ H.bf(w["router"]).astype(np.float64).T
    p = np.exp(logits - logits.max(1, keepdims=True))
    p /= p.sum(1, keepdims=True)
    deq = lambda m, r0, r1: H.bf(H.q4_dequant(m, slice(r0, r1))).astype(np.float64)  # noqa: E731
    silu = lambda v: v / (1.0 + np.exp(-v))  # noqa: E731
    ref = np.zeros((5, 128))
    for t in range(5):
        top = np.argsort(-p[t], kind="stable")[:3]
        wt = p[t, top] / p[t, top].sum()
        for e, we in zip(top, wt):
            g = deq(w["gate"], e * 64, (e + 1) * 64) @ xf[t]
            u = deq(w["up"], e * 64, (e + 1) * 64) @ xf[t]
            ref[t] += we * (deq(w["down"], e * 128, (e + 1) * 128) @ (silu(g) * u))
        gs = deq(w["sh_gate"], 0, 64) @ xf[t]
        us = deq(w["sh_up"], 0, 64) @ xf[t]
        ys = deq(w["sh_down"], 0, 128) @ (silu(gs) * us)
        ref[t] += ys / (1.0 + np.exp(-(xf[t] @ H.bf(w["shared_gate"]).astype(np.float64))))
    assert np.linalg.norm(got - ref) / np.linalg.norm(ref) < 2e-2
