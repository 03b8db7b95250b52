"""CPU tests of the oracle: pins against the reference kernel, closed forms, KATs."""
from __future__ import annotations

import numpy as np
import pytest

from conftest import rel_l2


def _rec_inputs(synth, B, T, hk, hv, dk=128, dv=128, seed=3, zero=False, g_lo=0.5):
    q = synth.normal_bf16(seed, "tq", (B, T, hk, dk), 0.05)
    kf = synth.normal(seed, "tk", B * T * hk * dk).reshape(B, T, hk, dk)
    kf = kf / np.linalg.norm(kf, axis=-1, keepdims=True)
    k = synth.f32_to_bf16(kf.astype(np.float32))
    v = synth.normal_bf16(seed, "tv", (B, T, hv, dv))
    g = synth.uniform(seed, "tg", B * T * hv, g_lo, 1.0).astype(np.float32).reshape(B, T, hv)
    beta = synth.f32_to_bf16(synth.uniform(seed, "tb", B * T * hv).astype(np.float32)).reshape(B, T, hv)
    st = np.zeros((B, hv, dv, dk), np.float32) if zero else \
        (synth.normal(seed, "ts", B * hv * dv * dk) * 0.1).astype(np.float32).reshape(B, hv, dv, dk)
    return q, k, v, g, beta, st


@pytest.mark.parametrize("shape", [(1, 1, 16, 32), (2, 5, 2, 4), (3, 4, 1, 2), (1, 9, 2, 2)])
def test_recurrence_bit_exact_vs_reference_kernel(oracle, synth, shape):
    """The oracle recurrence equals the reference's Metal kernel body run on the CPU, bit for bit."""
    if oracle.ref_lib() is None:
        pytest.skip("reference kernel CPU build absent (covered by the committed golden hashes)")
    B, T, hk, hv = shape
    args = _rec_inputs(synth, B, T, hk, hv)
    y1, s1 = oracle.recurrence(*args, T, B, hk, hv, 128, 128)
    y2, s2 = oracle.ref_recurrence(*args, T, B, hk, hv, 128, 128)
    assert np.array_equal(y1, y2)
    assert np.array_equal(s1.view(np.uint32), s2.view(np.uint32))


def test_recurrence_vs_f64(oracle, synth):
    """Independent float64 restatement of the algebra agrees to f32/bf16 precision."""
    B, T, hk, hv = 1, 6, 2, 4
    q, k, v, g, beta, st = _rec_inputs(synth, B, T, hk, hv)
    y, s = oracle.recurrence(q, k, v, g, beta, st, T, B, hk, hv, 128, 128)
    f = synth.bf16_to_f32
    y64, s64 = oracle.f64_recurrence(f(q[0]), f(k[0]), f(v[0]), g[0], f(beta[0]), st[0], hk, hv)
    assert rel_l2(s[0], s64) < 1e-5
    assert rel_l2(f(y[0]), y64) < 4e-3   # y is rounded to bf16


def test_closed_form_one_step_zero_state(oracle, synth):
    """From S=0, one step gives S = beta v k^T and y = beta v (k.q)."""
    B, T, hk, hv = 1, 1, 1, 2
    q, k, v, g, beta, st = _rec_inputs(synth, B, T, hk, hv, zero=True)
    y, s = oracle.recurrence(q, k, v, g, beta, st, T, B, hk, hv, 128, 128)
    f = synth.bf16_to_f32
    for h in range(hv):
        exp_s = f(beta[0, 0, h]) * np.outer(f(v[0, 0, h]).astype(np.float64), f(k[0, 0, 0]))
        assert rel_l2(s[0, h], exp_s) < 1e-6
        exp_y = exp_s @ f(q[0, 0, 0]).astype(np.float64)
        assert rel_l2(f(y[0, 0, h]), exp_y) < 4e-3


def test_beta_zero_is_pure_decay(oracle, synth):
    """With beta = 0 the state only decays: S_T = (prod g) S_0."""
    B, T, hk, hv = 1, 7, 1, 2
    q, k, v, g, beta, st = _rec_inputs(synth, B, T, hk, hv)
    beta = np.zeros_like(beta)
    _, s = oracle.recurrence(q, k, v, g, beta, st, T, B, hk, hv, 128, 128)
    for h in range(hv):
        assert rel_l2(s[0, h], np.prod(g[0, :, h].astype(np.float64)) * st[0, h]) < 1e-6


def test_delta_rule_overwrites_memory(oracle, synth):
    """g = 1, beta = 1 and a unit key: after the step S k = v exactly in exact arithmetic."""
    B, T, hk, hv = 1, 1, 1, 2
    q, k, v, g, beta, st = _rec_inputs(synth, B, T, hk, hv)
    g = np.ones_like(g)
    beta = np.full_like(beta, synth.f32_to_bf16(np.array([1.0], np.float32))[0])
    kk = np.zeros(128, np.float32)
    kk[17] = 1.0
    k = np.broadcast_to(synth.f32_to_bf16(kk), k.shape).copy()
    _, s = oracle.recurrence(q, k, v, g, beta, st, T, B, hk, hv, 128, 128)
    f = synth.bf16_to_f32
    for h in range(hv):
        assert rel_l2(s[0, h] @ kk, f(v[0, 0, h])) < 1e-6


def test_multi_token_equals_repeated_single_token(oracle, synth):
    """A T-token call of the recurrence equals T one-token calls, bit for bit."""
    B, T, hk, hv = 2, 5, 2, 4
    q, k, v, g, beta, st = _rec_inputs(synth, B, T, hk, hv)
    y_all, s_all = oracle.recurrence(q, k, v, g, beta, st, T, B, hk, hv, 128, 128)
    s = st
    ys = []
    for t in range(T):
        y1, s = oracle.recurrence(q[:, t:t + 1], k[:, t:t + 1], v[:, t:t + 1], g[:, t:t + 1], beta[:, t:t + 1], s,
                                  1, B, hk, hv, 128, 128)
        ys.append(y1)
    assert np.array_equal(np.concatenate(ys, axis=1), y_all)
    assert np.array_equal(s, s_all)


def test_packed_equals_dense(oracle, synth):
    """The packed ragged recurrence reproduces per-sequence dense calls."""
    hk, hv = 2, 4
    lens = [3, 1, 4]
    cu = np.concatenate([[0], np.cumsum(lens)]).astype(np.int32)
    N = int(cu[-1])
    q, k, v, g, beta, _ = _rec_inputs(synth, 1, N, hk, hv)
    st = (synth.normal(9, "pk", len(lens) * hv * 128 * 128) * 0.1).astype(np.float32).reshape(len(lens), hv, 128, 128)
    y, s = oracle.recurrence_packed(q[0], k[0], v[0], g[0], beta[0], st, cu, hk, hv, 128, 128)
    for i, T in enumerate(lens):
        a, b = cu[i], cu[i + 1]
        yd, sd = oracle.recurrence(q[:, a:b], k[:, a:b], v[:, a:b], g[:, a:b], beta[:, a:b], st[i:i + 1], T, 1, hk,
                                   hv, 128, 128)
        assert np.array_equal(y[a:b], yd[0])
        assert np.array_equal(s[i], sd[0])


def test_gates_formula(oracle, synth):
    hv = 32
    ab = synth.normal_bf16(1, "gab", (10, 2 * hv))
    A_log = synth.uniform(1, "A", hv, 0.0, np.log(16.0)).astype(np.float32)
    dt = synth.uniform(1, "dt", hv, -1, 1).astype(np.float32)
    g, beta = oracle.gates(ab, A_log, dt, hv)
    f = synth.bf16_to_f32
    b = f(ab[:, :hv]).astype(np.float64)
    a = f(ab[:, hv:]).astype(np.float64)
    beta_ref = 1.0 / (1.0 + np.exp(-b))
    g_ref = np.exp(-np.exp(A_log.astype(np.float64)) * np.log1p(np.exp(a + dt)))
    assert np.max(np.abs(f(beta) - beta_ref)) <= 2.0 ** -8
    assert rel_l2(g, g_ref) < 1e-5
    assert np.all((g > 0) & (g < 1))


def test_gates_bf16_dt_bias_rounds_the_add_and_exp(oracle, synth):
    """A checkpoint that stores dt_bias in bf16: MLX adds a_raw + dt_bias and exponentiates in bf16
    (compiled_ops.rs:36-37), then adds the f32 constant 1 in f32 (:38-39).  The oracle's bf16 mode equals
    that two-rounding restatement and differs from the f32 mode."""
    hv = 32
    ab = synth.normal_bf16(2, "gab16", (64, 2 * hv))
    A_log = synth.uniform(2, "A", hv, 0.0, np.log(16.0)).astype(np.float32)
    dt = synth.bf16_to_f32(synth.f32_to_bf16(synth.uniform(2, "dt", hv, -1, 1).astype(np.float32)))
    g16, beta16 = oracle.gates(ab, A_log, dt, hv, dt_bias_bf16=True)
    g32, beta32 = oracle.gates(ab, A_log, dt, hv)
    f = synth.bf16_to_f32
    r = lambda x: f(synth.f32_to_bf16(np.asarray(x, np.float32)))
    a = f(ab[:, hv:])
    s = r(a + dt[None, :])
    es = r(np.exp(s.astype(np.float64)).astype(np.float32))
    sp = np.log(es.astype(np.float64) + 1.0)
    g_ref = np.exp(-np.exp(A_log.astype(np.float64)) * sp)
    assert rel_l2(g16, g_ref) < 1e-6
    assert np.array_equal(beta16, beta32)            # beta does not involve dt_bias
    assert np.count_nonzero(g16 != g32) > g16.size // 4   # the two roundings change most gates


def test_conv_one_hot_tap_kat(oracle, synth):
    """A conv weight with a single 1.0 tap returns silu of the tap-shifted input, on both rounding paths."""
    cfg = synth.GdnConfig(n_layers=1)
    D = cfg.conv_dim
    one = synth.f32_to_bf16(np.array([1.0], np.float32))[0]
    f = synth.bf16_to_f32
    for T in (1, 6):
        x = synth.normal_bf16(2, "katx", (T, D))
        cs0 = synth.normal_bf16(2, "katcs", (3, D))
        padded = np.concatenate([cs0, x])
        for tap in range(4):
            cw = np.zeros((D, 4), np.uint16)
            cw[:, tap] = one
            out, cs = oracle.conv(cfg, x, cs0, cw)
            xs = f(padded[tap:tap + T]).astype(np.float32)
            exp = synth.f32_to_bf16((xs * (np.float32(1) / (np.float32(1) + np.exp(-xs)))).astype(np.float32))
            assert np.max(np.abs(f(out).astype(np.float64) - f(exp))) <= 2.0 ** -7 * np.max(np.abs(f(exp))) + 1e-30
            assert np.array_equal(cs, padded[-3:])    # new state = last 3 rows of [state; x]


def test_conv_decode_and_prefill_rounding_differ_only_in_conv(oracle, synth):
    """T one-token layer steps vs one T-token step: same result up to the reference's conv rounding split."""
    cfg = synth.GdnConfig(n_layers=1)
    w = synth.layer_weights(cfg, 0, with_proj=False)
    T = 4
    inp = synth.step_inputs(cfg, T, seed=5, tag="split")
    conv0, rec0 = synth.random_states(cfg, 1, seed=5, tag="split")
    out_p, cs_p, rs_p, _ = oracle.layer_step(cfg, w, inp["qkv"], inp["z"], inp["ab"], conv0, rec0,
                                             np.array([0, T], np.int32))
    cs, rs = conv0, rec0
    outs = []
    for t in range(T):
        o, cs, rs, _ = oracle.layer_step(cfg, w, inp["qkv"][t:t + 1], inp["z"][t:t + 1], inp["ab"][t:t + 1], cs, rs,
                                         np.array([0, 1], np.int32))
        outs.append(o)
    assert np.array_equal(cs, cs_p)                        # conv state: exact copy of inputs either way
    assert rel_l2(rs, rs_p) < 2e-2                         # differs only through bf16 conv rounding
    assert rel_l2(synth.bf16_to_f32(np.concatenate(outs)), synth.bf16_to_f32(out_p)) < 5e-2


def test_stack_step_runs(oracle, synth):
    """The residual stack step composes layers: two 1-layer calls == one 2-layer call."""
    cfg = synth.GdnConfig(hidden=256, n_k_heads=2, n_v_heads=4, n_layers=2)
    ws = [synth.layer_weights(cfg, l) for l in range(2)]
    h0 = synth.normal_bf16(0, "stk", (3, cfg.hidden))
    cu = np.array([0, 1, 3], np.int32)
    L, n = 2, 2
    cs0 = np.zeros((L, n, 3, cfg.conv_dim), np.uint16)
    rs0 = np.zeros((L, n, cfg.hv, 128, 128), np.float32)
    h2, cs2, rs2 = oracle.stack_step(cfg, ws, h0, cs0, rs0, cu)
    h1, a_cs, a_rs = oracle.stack_step(cfg, ws[:1], h0, cs0[:1], rs0[:1], cu)
    h1, b_cs, b_rs = oracle.stack_step(cfg, ws[1:], h1, cs0[1:], rs0[1:], cu)
    assert np.array_equal(h1, h2)
    assert np.array_equal(np.concatenate([a_rs, b_rs]), rs2)
